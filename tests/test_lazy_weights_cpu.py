"""Random-init weights drawn as the model takes them: the same values as the
eager draw, and with quantised experts each MoE layer quantises its bf16
experts before the next layer's are drawn (what lets a Kimi-K2-shape model
load on 180 GB GPUs: one layer of bf16 experts at a time, not all of them)."""

import torch

from minisgl.engine.config import EngineConfig
from minisgl.models import LazyRandomWeights, create_model, random_weights
from minisgl.parallel import DistributedInfo, info
from minisgl.utils import torch_dtype
from minisgl.utils.synthetic import make_model_dir


def _meta_model(quant: str, monkeypatch):
    # the engine sets this once per process; restored after the test
    monkeypatch.setattr(info, "_TP", DistributedInfo(0, 1))
    cfg = EngineConfig(model_path=make_model_dir("tiny-qwen3-moe"), tp_info=DistributedInfo(0, 1),
                       dtype=torch.float32, device="cpu", moe_quant=quant)
    with torch.device("meta"), torch_dtype(torch.float32):
        return create_model(cfg.model_config)


def test_lazy_draw_gives_the_eager_values(monkeypatch):
    shapes = _meta_model("none", monkeypatch).state_dict()
    eager = random_weights(shapes, torch.device("cpu"), seed=3)
    lazy = LazyRandomWeights(shapes, torch.device("cpu"), seed=3)
    assert sorted(lazy) == sorted(eager) and len(lazy) == len(eager)
    for name in sorted(eager)[::3]:  # in another order than the eager draw
        assert torch.equal(lazy.pop(name), eager[name]), name
    assert lazy.pop("no.such.weight", None) is None


def test_experts_are_quantised_layer_by_layer(monkeypatch):
    model = _meta_model("mxfp4", monkeypatch)
    layers = model.model.layers.op_list
    shapes = model.state_dict()
    seen = []

    class Watch(LazyRandomWeights):
        def pop(self, name, *default):
            if name.endswith("experts.gate_up_proj"):
                seen.append((int(name.split(".")[2]), [dl.mlp.experts._mxfp4 is not None for dl in layers]))
            return super().pop(name, *default)

    model.load_state_dict(Watch(shapes, torch.device("cpu"), seed=3))
    assert [i for i, _ in seen] == list(range(len(layers)))
    for i, done in seen:
        assert done == [j < i for j in range(len(layers))], (i, done)
    assert all(dl.mlp.experts._mxfp4 is not None for dl in layers)
