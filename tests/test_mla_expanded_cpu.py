"""The non-absorbed MLA prefill on the CPU (every key's c_kv expanded
through kv_b_proj, then attention with 192-dim scores and 128-dim values in
the real shapes; tiny dims here), forced for every prefill batch: the
engine must reproduce the dense fp32 oracle; and the expanded form equals the
absorbed one op for op."""

import random

import torch

from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl.models.oracle import greedy_generate
from minisgl.ops import reference as ref
from minisgl.utils.synthetic import make_model_dir


def test_expanded_prefill_matches_dense_mla_oracle(monkeypatch):
    """Prefill through the non-absorbed form (every key expanded through
    kv_b_proj), forced for every prefill batch; decode stays absorbed."""
    monkeypatch.setenv("MINISGL_MLA_PREFILL", "expanded")
    d = make_model_dir("tiny-kimi")
    engine = LLM(d, dtype=torch.float32, device="cpu", use_dummy_weight=True, page_size=16, max_extend_tokens=32,
                 num_page_override=128, max_running_req=8, max_seq_len_override=512, cache_type="radix")
    try:
        rng = random.Random(5)
        prompts = [[rng.randrange(1024) for _ in range(rng.randint(8, 70))] for _ in range(4)]
        outs = engine.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
        model = engine.engine.model
        for p, o in zip(prompts, outs):
            assert o["token_ids"] == greedy_generate(model.state_dict(), engine.engine.model_config, p, 6)
    finally:
        engine.shutdown()


def test_expanded_equals_absorbed_attention():
    g = torch.Generator().manual_seed(2)
    H, nope, rope, v, kv_lora, page = 3, 16, 8, 12, 32, 16
    lens, qlens = [5, 40, 33], [5, 7, 33]
    pages = sum((L + page - 1) // page for L in lens) + 1
    latent = torch.randn(pages, page, kv_lora + rope, generator=g)
    pt = torch.zeros(len(lens), 64, dtype=torch.int32)
    nxt = 1
    for b, L in enumerate(lens):
        for p in range(L):
            if p % page == 0:
                nxt += 1
            pt[b, p] = (nxt - 1) * page + p % page
    rows = torch.arange(len(lens), dtype=torch.int32)
    seq = torch.tensor(lens, dtype=torch.int32)
    cu = torch.tensor([0] + torch.tensor(qlens).cumsum(0).tolist(), dtype=torch.int32)
    T = sum(qlens)
    q = torch.randn(T, H, nope + rope, generator=g)
    q_rope = torch.randn(T, H, rope, generator=g)
    w = torch.randn(H * (nope + v), kv_lora, generator=g) * 0.2
    scale = 0.3
    got = ref.mla_prefill_attention(q, q_rope, latent, pt, rows, seq, cu, w, kv_lora, nope, v, page, scale)
    # absorbed: q_lat = q_nope W_UK, scores against [c_kv | k_rope], output through W_UV
    wv = w.view(H, nope + v, kv_lora)
    q_lat = torch.einsum("thn,hnc->htc", q[..., :nope], wv[:, :nope])
    o_lat = ref.mla_attention(q_lat, q_rope, latent, pt, rows, seq, cu, page, scale)
    want = torch.einsum("htc,hvc->thv", o_lat, wv[:, nope:]).reshape(T, H * v)
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-4)
