"""The whole server on the CPU, end to end over HTTP.

`python -m minisgl --model synthetic:<shape> --device cpu` starts the API
process, the tokenizer / detokenizer and the scheduler ranks. The test calls:

- /v1/models;
- /v1/chat/completions, plain and streamed (SSE);
- /generate (streamed);
- the online benchmark client (minisgl/benchmark/online.py), a short run and a trace replay;
- a client that disconnects mid-stream (its request is aborted, serving goes on).

It checks the response formats and the token counts. Greedy requests must be
repeatable. The server's process group is killed at the end (it was started
in its own session, so only its processes are signalled).
"""

import json
import os
import signal
import socket
import subprocess
import sys
import time
import urllib.error
import urllib.request

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    while True:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        with socket.socket() as s2:  # the server also binds port + 1 for its process group
            try:
                s2.bind(("127.0.0.1", port + 1))
                return port
            except OSError:
                continue


def _post(url, body, timeout=120):
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    return urllib.request.urlopen(req, timeout=timeout)


def _sse_payloads(resp):
    out = []
    for raw in resp:
        line = raw.decode().rstrip("\n")
        if line.startswith("data: "):
            out.append(line[len("data: "):])
    return out


# 0 extra tokenizers: the detokenizer also tokenizes; 1: a separate tokenizer process; the MoE case runs two
# ranks with DP attention (each rank serves its own requests, experts split over the ranks)
@pytest.mark.parametrize("model,extra", [("tiny-qwen3", ["--num-tokenizer", "0"]),
                                         ("tiny-qwen3", ["--num-tokenizer", "1"]),
                                         ("tiny-qwen3-moe", ["--tp", "2", "--enable-dp-attention"])],
                         ids=["shared-tokenizer", "separate-tokenizer", "tp2-dp-attention"])
def test_http_server_end_to_end(tmp_path, model, extra):
    port = _free_port()
    base = f"http://127.0.0.1:{port}"
    log_path = tmp_path / "server.log"
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    with open(log_path, "w") as log:
        proc = subprocess.Popen([sys.executable, "-m", "minisgl", "--model", f"synthetic:{model}", "--device", "cpu",
                                 "--port", str(port), "--max-running-requests", "4", "--max-seq-len-override", "256",
                                 "--num-pages", "64", "--page-size", "16"] + extra,
                                cwd=ROOT, env=env, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
    try:
        deadline = time.monotonic() + 300
        while True:
            assert proc.poll() is None, "server exited:\n" + log_path.read_text()[-3000:]
            assert time.monotonic() < deadline, "server not ready:\n" + log_path.read_text()[-3000:]
            try:
                with urllib.request.urlopen(base + "/v1/models", timeout=5) as r:
                    models = json.load(r)
                break
            except (urllib.error.URLError, ConnectionError, OSError):
                time.sleep(1)
        assert models["data"] and models["data"][0]["id"]

        chat = {"model": "tiny", "messages": [{"role": "user", "content": "hello there"}], "max_tokens": 5,
                "temperature": 0.0, "ignore_eos": True}
        with _post(base + "/v1/chat/completions", chat) as r:
            first = json.load(r)
        assert first["object"] == "chat.completion"
        assert first["choices"][0]["message"]["role"] == "assistant"
        assert first["usage"]["completion_tokens"] == 5
        with _post(base + "/v1/chat/completions", chat) as r:
            again = json.load(r)
        assert again["choices"][0]["message"]["content"] == first["choices"][0]["message"]["content"]

        with _post(base + "/v1/chat/completions", dict(chat, stream=True)) as r:
            payloads = _sse_payloads(r)
        assert payloads[-1] == "[DONE]"
        chunks = [json.loads(p) for p in payloads[:-1]]
        assert chunks[0]["choices"][0]["delta"].get("role") == "assistant"
        assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
        streamed = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks)
        assert streamed == first["choices"][0]["message"]["content"]

        with _post(base + "/generate", {"prompt": "hello there", "max_tokens": 4, "ignore_eos": True}) as r:
            payloads = _sse_payloads(r)
        assert payloads[-1] == "[DONE]" and len(payloads) == 4 + 1

        if extra == ["--num-tokenizer", "0"]:  # the online benchmark client against this server
            import asyncio

            from minisgl.benchmark import online

            res = asyncio.run(online.run(base, num_requests=6, concurrency=3, input_len=12, output_len=5))
            assert res["completed"] == 6 and res["output_tokens"] == 30, res
            for key in ("ttft_ms", "tpot_ms", "e2e_ms"):
                st = res[key]
                assert 0 < st["p50"] <= st["max"] and st["avg"] > 0, (key, st)
            assert res["ttft_ms"]["max"] <= res["e2e_ms"]["max"]
            trace = tmp_path / "trace.jsonl"
            trace.write_text("".join(json.dumps({"timestamp": t, "input_length": 10, "output_length": 3}) + "\n"
                                     for t in (0, 200, 400)))  # Mooncake format: milliseconds
            res = asyncio.run(online.run_trace(base, online.read_trace(str(trace), "mooncake")))
            assert res["completed"] == 3 and res["output_tokens"] == 9 and res["wall_s"] >= 0.4, res
            # per-request output lengths, Poisson arrivals (one point of a rate sweep)
            res = asyncio.run(online.run_requests(base, ["alpha beta gamma"] * 4, [2, 3, 4, 5], 4,
                                                  request_rate=20.0, input_lens=[3] * 4))
            assert res["completed"] == 4 and res["output_tokens"] == 14, res

            # a client that leaves mid-stream: the server aborts its request and keeps serving
            import http.client

            conn = http.client.HTTPConnection("127.0.0.1", port, timeout=60)
            conn.request("POST", "/v1/chat/completions", body=json.dumps(dict(chat, max_tokens=240, stream=True)),
                         headers={"Content-Type": "application/json"})
            resp = conn.getresponse()
            got = 0
            while got < 2:
                if resp.readline().startswith(b"data: "):
                    got += 1
            conn.close()
            deadline = time.monotonic() + 60
            while "aborting request" not in log_path.read_text():
                assert time.monotonic() < deadline, "no abort after the disconnect:\n" + log_path.read_text()[-3000:]
                time.sleep(0.2)
            with _post(base + "/v1/chat/completions", chat) as r:
                assert json.load(r)["usage"]["completion_tokens"] == 5
    finally:
        try:
            os.killpg(proc.pid, signal.SIGTERM)
            proc.wait(timeout=30)
        except (ProcessLookupError, subprocess.TimeoutExpired):
            try:
                os.killpg(proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            proc.wait(timeout=30)


def test_shell_mode_answers_and_exits(tmp_path):
    """`--shell` reads lines from standard input, prints each answer, and
    leaves on /exit with its worker processes stopped."""
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""),
               MINISGL_SHELL_MAX_TOKENS="4", MINISGL_SHELL_TEMPERATURE="0")
    proc = subprocess.Popen([sys.executable, "-m", "minisgl", "--model", "synthetic:tiny-qwen3", "--device", "cpu",
                             "--port", str(_free_port()), "--max-seq-len-override", "256", "--num-pages", "64",
                             "--page-size", "16", "--shell"],
                            cwd=ROOT, env=env, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                            stderr=subprocess.STDOUT, start_new_session=True)
    try:
        out, _ = proc.communicate(b"hello there\n/reset\n/bogus\n/exit\n", timeout=300)
    finally:
        if proc.poll() is None:
            os.killpg(proc.pid, signal.SIGKILL)
            proc.wait(timeout=30)
    text = out.decode(errors="replace")
    assert "unknown command /bogus" in text, text[-3000:]
    assert "Exiting shell..." in text, text[-3000:]
