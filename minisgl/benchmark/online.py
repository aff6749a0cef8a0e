"""Online serving benchmark: streamed chat completions against a running server.

    python -m minisgl.benchmark.online --url http://127.0.0.1:1919 \\
        --num-requests 64 --concurrency 16 --input-len 256 --output-len 128 [--tokenizer PATH]

Each request streams `/v1/chat/completions` (greedy, `ignore_eos`) and records:

- TTFT: request sent -> first token chunk;
- TPOT: (last token - first token) / (tokens - 1);
- end-to-end latency.

At most `--concurrency` requests are in flight; with `--request-rate R` new ones
also start as a Poisson process of R per second.

One JSON line reports avg / p50 / p90 / p99 / max of each metric, plus output and
input tokens per second over the whole run. These are the client-side metrics of the
reference's client (python/minisgl/benchmark/client.py:320-384), measured with
aiohttp instead of the openai package.

Prompts are random token ids decoded by `--tokenizer` (a model folder), so a prompt
holds about `--input-len` tokens. Without a tokenizer they are random words.

`--workload qwen3-32b` (or another pool of minisgl.benchmark.workload) sends
that pool instead: lognormal prompt and output lengths, 30 % of the prompts
behind one of 50 shared prefixes (the same text, so the server's radix cache
serves them). `--rate-sweep 0.5,1,2,4` runs the requests once per Poisson
rate, without a concurrency cap, and prints one line per rate: the
throughput / TTFT / TPOT curve of an online serving benchmark.

`--trace FILE --trace-format {qwen,mooncake}` replays a request trace instead. Both
formats are JSON lines with `timestamp`, `input_length` and `output_length`; other
fields are ignored. Timestamps are seconds in Qwen traces and milliseconds in Mooncake
traces, as in the reference's readers (python/minisgl/benchmark/client.py:407-495).
Each request starts at its offset from the first one, times `--trace-scale`, with no
concurrency cap.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

_WORDS = ("the of and to in is was for on as with by at from that this which be are an or it not have "
          "time year people way day man thing woman life child world school state family student group "
          "country problem hand part place case week company system program question work government").split()


@dataclass
class RequestResult:
    ok: bool
    prompt_chars: int
    tokens: int = 0
    ttft: float = 0.0
    e2e: float = 0.0
    token_times: List[float] = field(default_factory=list)
    error: str = ""

    @property
    def tpot(self) -> Optional[float]:
        if self.tokens < 2:
            return None
        return (self.token_times[-1] - self.token_times[0]) / (self.tokens - 1)


def make_prompts(n: int, input_len: int, tokenizer_path: Optional[str], seed: int) -> List[str]:
    rng = random.Random(seed)
    if tokenizer_path:
        from minisgl.utils import load_tokenizer

        tok = load_tokenizer(tokenizer_path)
        vocab = getattr(tok, "vocab_size", 32000)
        return [tok.decode([rng.randrange(100, max(101, vocab - 100)) for _ in range(input_len)]) for _ in range(n)]
    return [" ".join(rng.choice(_WORDS) for _ in range(input_len)) for _ in range(n)]


def pool_prompts(shape: str, n: int, tokenizer_path: Optional[str], seed: int):
    """(prompt texts, output lengths, prompt lengths in pool tokens) of a
    minisgl.benchmark.workload pool.
    Token ids become text through the tokenizer (ids moved clear of the
    special ids at the bottom of the vocabulary) or as words; equal id
    prefixes give equal text prefixes."""
    from minisgl.benchmark.workload import make_pool

    ids, outs = make_pool(shape, n, seed)
    if tokenizer_path:
        from minisgl.utils import load_tokenizer

        tok = load_tokenizer(tokenizer_path)
        span = max(1, getattr(tok, "vocab_size", 32000) - 200)
        texts = [tok.decode([100 + t % span for t in p]) for p in ids]
    else:
        texts = [" ".join(_WORDS[t % len(_WORDS)] for t in p) for p in ids]
    return texts, outs, [len(p) for p in ids]


async def _one(session, url: str, model: str, prompt: str, output_len: int, timeout: float) -> RequestResult:
    import aiohttp

    body = {"model": model, "messages": [{"role": "user", "content": prompt}], "max_tokens": output_len,
            "temperature": 0.0, "ignore_eos": True, "stream": True}
    res = RequestResult(ok=False, prompt_chars=len(prompt))
    t0 = time.perf_counter()
    try:
        async with session.post(url + "/v1/chat/completions", json=body,
                                timeout=aiohttp.ClientTimeout(total=timeout)) as resp:
            if resp.status != 200:
                res.error = f"HTTP {resp.status}: {(await resp.text())[:200]}"
                return res
            async for raw in resp.content:
                line = raw.decode().strip()
                if not line.startswith("data: "):
                    continue
                data = line[len("data: "):]
                if data == "[DONE]":
                    break
                choice = json.loads(data)["choices"][0]
                if choice.get("finish_reason") is not None:
                    continue  # the closing chunk carries no token
                now = time.perf_counter() - t0
                if not res.token_times:
                    res.ttft = now
                res.token_times.append(now)
        res.tokens = len(res.token_times)
        res.e2e = time.perf_counter() - t0
        res.ok = res.tokens > 0
        if not res.ok:
            res.error = "no tokens"
    except Exception as e:  # one failed request is reported, not fatal
        res.error = f"{type(e).__name__}: {e}"
    return res


@dataclass
class TraceEntry:
    start_s: float  # offset from the first request (after scaling)
    input_len: int
    output_len: int


def read_trace(path: str, fmt: str, n: Optional[int] = None, scale: float = 1.0) -> List[TraceEntry]:
    """Requests of a Qwen (seconds) or Mooncake (milliseconds) JSON-lines trace, sorted by start."""
    if fmt not in ("qwen", "mooncake"):
        raise ValueError(f"unknown trace format {fmt!r} (qwen or mooncake)")
    unit = 1.0 if fmt == "qwen" else 1e-3
    rows = []
    with open(path) as f:
        for line in f:
            if not line.strip():
                continue
            obj = json.loads(line)
            rows.append((float(obj["timestamp"]) * unit, int(obj["input_length"]), int(obj["output_length"])))
            if n is not None and len(rows) >= n:
                break
    if not rows:
        return []
    t0 = min(r[0] for r in rows)
    return sorted((TraceEntry((t - t0) * scale, i, o) for t, i, o in rows), key=lambda e: e.start_s)


def _stats(xs: List[float]) -> Dict[str, float]:
    if not xs:
        return {}
    s = sorted(xs)

    def pct(p: float) -> float:
        return s[min(len(s) - 1, int(round(p / 100.0 * (len(s) - 1))))]

    return {"avg": round(sum(s) / len(s) * 1e3, 3), "p50": round(pct(50) * 1e3, 3), "p90": round(pct(90) * 1e3, 3),
            "p99": round(pct(99) * 1e3, 3), "max": round(s[-1] * 1e3, 3)}


def summarize(results: List[RequestResult], wall: float, input_len: int,
              input_lens: Optional[List[int]] = None) -> Dict[str, object]:
    ok = [r for r in results if r.ok]
    in_tokens = (sum(n for r, n in zip(results, input_lens) if r.ok) if input_lens is not None
                 else len(ok) * input_len)
    out_tokens = sum(r.tokens for r in ok)
    tpots = [t for t in (r.tpot for r in ok) if t is not None]
    return {"bench": "online", "requests": len(results), "completed": len(ok),
            "errors": sorted({r.error for r in results if not r.ok})[:5],
            "wall_s": round(wall, 3), "output_tokens": out_tokens,
            "output_tok_per_s": round(out_tokens / wall, 1) if wall > 0 else 0.0,
            "input_tok_per_s": round(in_tokens / wall, 1) if wall > 0 else 0.0,
            "ttft_ms": _stats([r.ttft for r in ok]), "tpot_ms": _stats(tpots), "e2e_ms": _stats([r.e2e for r in ok])}


async def run(url: str, num_requests: int, concurrency: int, input_len: int, output_len: int,
              request_rate: float = float("inf"), tokenizer: Optional[str] = None, seed: int = 0,
              timeout: float = 600.0) -> Dict[str, object]:
    prompts = make_prompts(num_requests, input_len, tokenizer, seed)
    return await run_requests(url, prompts, [output_len] * len(prompts), concurrency, request_rate, seed, timeout,
                              input_len=input_len)


async def run_requests(url: str, prompts: List[str], output_lens: List[int], concurrency: int,
                       request_rate: float = float("inf"), seed: int = 0, timeout: float = 600.0,
                       input_len: int = 0, input_lens: Optional[List[int]] = None) -> Dict[str, object]:
    """Send the prompts (at most ``concurrency`` in flight; with a finite
    ``request_rate`` starting as a Poisson process) and summarise."""
    import aiohttp

    rng = random.Random(seed + 1)
    sem = asyncio.Semaphore(max(1, concurrency))
    async with aiohttp.ClientSession() as session:
        async with session.get(url + "/v1/models") as resp:
            model = (await resp.json())["data"][0]["id"]

        async def guarded(p: str, n_out: int) -> RequestResult:
            async with sem:
                return await _one(session, url, model, p, n_out, timeout)

        t0 = time.perf_counter()
        tasks = []
        for p, n_out in zip(prompts, output_lens):
            tasks.append(asyncio.create_task(guarded(p, n_out)))
            if request_rate != float("inf"):
                await asyncio.sleep(rng.expovariate(request_rate))
        results = await asyncio.gather(*tasks)
        wall = time.perf_counter() - t0
    return summarize(list(results), wall, input_len, input_lens)


def parse_rates(text: str) -> List[float]:
    """"0.5,1,2" -> [0.5, 1.0, 2.0]; "inf" allowed."""
    rates = [float(x) for x in text.split(",") if x.strip()]
    if not rates or any(r <= 0 for r in rates):
        raise ValueError(f"request rates must be positive: {text!r}")
    return rates


async def run_trace(url: str, entries: List[TraceEntry], tokenizer: Optional[str] = None, seed: int = 0,
                    timeout: float = 600.0) -> Dict[str, object]:
    import aiohttp

    prompts = [make_prompts(1, e.input_len, tokenizer, seed + i)[0] for i, e in enumerate(entries)]
    async with aiohttp.ClientSession() as session:
        async with session.get(url + "/v1/models") as resp:
            model = (await resp.json())["data"][0]["id"]
        t0 = time.perf_counter()

        async def timed(e: TraceEntry, prompt: str) -> RequestResult:
            await asyncio.sleep(max(0.0, t0 + e.start_s - time.perf_counter()))
            return await _one(session, url, model, prompt, e.output_len, timeout)

        results = await asyncio.gather(*(timed(e, p) for e, p in zip(entries, prompts)))
        wall = time.perf_counter() - t0
    out = summarize(list(results), wall, 0, [e.input_len for e in entries])
    out["bench"] = "online_trace"
    return out


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--url", default="http://127.0.0.1:1919")
    p.add_argument("--num-requests", type=int, default=64)
    p.add_argument("--concurrency", type=int, default=16)
    p.add_argument("--input-len", type=int, default=256)
    p.add_argument("--output-len", type=int, default=128)
    p.add_argument("--request-rate", type=float, default=float("inf"), help="requests per second (Poisson)")
    p.add_argument("--tokenizer", default=None, help="model folder whose tokenizer builds the prompts")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--trace", default=None, help="JSON-lines request trace to replay")
    p.add_argument("--trace-format", default="qwen", choices=["qwen", "mooncake"])
    p.add_argument("--trace-scale", type=float, default=1.0, help="multiplies the trace's time offsets")
    p.add_argument("--workload", default="fixed",
                   help="fixed (--input-len / --output-len) or a pool of minisgl.benchmark.workload: qwen3-32b, "
                        "qwen3-0.6b, kimi-k2")
    p.add_argument("--rate-sweep", default=None, help="comma-separated Poisson rates (req/s), one run and line each")
    args = p.parse_args()
    url = args.url.rstrip("/")
    if args.workload != "fixed" or args.rate_sweep:
        if args.workload == "fixed":
            prompts = make_prompts(args.num_requests, args.input_len, args.tokenizer, args.seed)
            outs, in_lens = [args.output_len] * len(prompts), [args.input_len] * len(prompts)
        else:
            prompts, outs, in_lens = pool_prompts(args.workload, args.num_requests, args.tokenizer, args.seed)
        rates = parse_rates(args.rate_sweep) if args.rate_sweep else [args.request_rate]
        for rate in rates:
            # a sweep point is an open-loop Poisson run: no concurrency cap
            conc = len(prompts) if args.rate_sweep else args.concurrency
            out = asyncio.run(run_requests(url, prompts, outs, conc, rate, args.seed, input_lens=in_lens,
                                           input_len=args.input_len))
            out.update(workload=args.workload, request_rate=rate)
            print(json.dumps(out), flush=True)
        return
    if args.trace:
        entries = read_trace(args.trace, args.trace_format, args.num_requests, args.trace_scale)
        out = asyncio.run(run_trace(url, entries, args.tokenizer, args.seed))
    else:
        out = asyncio.run(run(url, args.num_requests, args.concurrency, args.input_len, args.output_len,
                              args.request_rate, args.tokenizer, args.seed))
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
