"""Process topology: N scheduler ranks (one per GPU), one detokenizer (also
the tokenizer by default), optional extra tokenizers, and the API process
(python/minisgl/server/launch.py in the reference)."""

from __future__ import annotations

import logging
import multiprocessing as mp
import sys
from dataclasses import replace
from typing import TYPE_CHECKING

from minisgl.parallel import DistributedInfo
from minisgl.utils import init_logger

if TYPE_CHECKING:
    from .args import ServerArgs


def _run_scheduler(args: "ServerArgs", ack_queue) -> None:
    import torch

    from minisgl.scheduler import Scheduler

    with torch.inference_mode():
        scheduler = Scheduler(args)
        scheduler.sync_all_ranks()
        if args.tp_info.is_primary():
            ack_queue.put("Scheduler is ready")
        if args.silent_output:
            logging.disable(logging.INFO)
        try:
            scheduler.run_forever()
        except KeyboardInterrupt:
            if args.tp_info.is_primary():
                init_logger(__name__).info("Scheduler exiting gracefully...")
            scheduler.shutdown()


def start_backend_processes(server_args: "ServerArgs") -> list:
    from minisgl.tokenizer import tokenize_worker

    ctx = mp.get_context("spawn")
    ack = ctx.Queue()
    procs = []
    world = server_args.tp_info.size
    for rank in range(world):
        p = ctx.Process(target=_run_scheduler, args=(replace(server_args, tp_info=DistributedInfo(rank, world)), ack),
                        name=f"minisgl-TP{rank}-scheduler", daemon=False)
        p.start()
        procs.append(p)
    n_tok = server_args.num_tokenizer
    common = dict(tokenizer_path=server_args.model_path, backend_addr=server_args.zmq_backend_addr,
                  frontend_addr=server_args.zmq_frontend_addr, local_bs=1,
                  create=server_args.tokenizer_create_addr, ack_queue=ack)
    p = ctx.Process(target=tokenize_worker, kwargs=dict(common, addr=server_args.zmq_detokenizer_addr,
                                                        tokenizer_id=n_tok), name="minisgl-detokenizer-0")
    p.start()
    procs.append(p)
    for i in range(n_tok):
        p = ctx.Process(target=tokenize_worker, kwargs=dict(common, addr=server_args.zmq_tokenizer_addr,
                                                            tokenizer_id=i), name=f"minisgl-tokenizer-{i}")
        p.start()
        procs.append(p)
    logger = init_logger(__name__, "initializer")
    for _ in range(n_tok + 2):  # primary scheduler + detokenizer + tokenizers
        logger.info(ack.get())
    return procs


def launch_server(run_shell: bool = False) -> None:
    from .api_server import run_api_server
    from .args import parse_args

    server_args, run_shell = parse_args(sys.argv[1:], run_shell)
    run_api_server(server_args, lambda: start_backend_processes(server_args), run_shell=run_shell)


if __name__ == "__main__":
    launch_server()
