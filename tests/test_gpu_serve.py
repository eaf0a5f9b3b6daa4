"""g4_serve, the reference engine's process interface (gemma4_engine.cpp:1681-1689, as
server/server.py:44-75 drives it), run as a subprocess on the synthetic model at reduced size: the
server's handshake ("0 2"), requests that reuse a prefix, BENCH_MODE, the streamed FIRST / TOK
lines, GEN and TIMING.  The tokens must equal the request policy restated over oracle models
(tests/test_gpu_requests.py), with k changed by BENCH_MODE on both sides."""
import os
import pathlib
import subprocess

import numpy as np
import pytest

from oracle_lib import make_prompt
from test_gpu_requests import SMALL, OracleConversations

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BIN = pathlib.Path(__file__).resolve().parent.parent / "gemma4-e2b-laptop-cpu_b200" / "g4_serve"


def _env():
    env = dict(os.environ)
    env.update(ENGINE_SERVE="1", ENGINE_STREAM="1", G4_HIDDEN=str(SMALL["hidden"]), G4_LAYERS=str(SMALL["n_layers"]),
               G4_MLP=str(SMALL["mlp"]), G4_VOCAB=str(SMALL["vocab"]), ENGINE_CTX=str(SMALL["ctx_max"]),
               ENGINE_PREFILL_INT8="1", ENGINE_NGRAM="2", ENGINE_K="3")
    return env


def _parse(lines):
    """Responses in order: ("req", first, streamed, gen, timing) or ("mode", line) / ("audio", line)."""
    out, cur = [], None
    for ln in lines:
        if ln.startswith("FIRST "):
            cur = {"first": int(ln.split()[1]), "tok": []}
        elif ln.startswith("TOK"):
            cur["tok"] += [int(x) for x in ln.split()[1:]]
        elif ln.startswith("GEN:"):
            gen = [int(x) for x in ln.split()[1:]]
            cur = cur or {"first": None, "tok": []}
            cur["gen"] = gen
        elif ln.startswith("TIMING "):
            cur["timing"] = dict(kv.split("=", 1) for kv in ln.split()[1:] if "=" in kv)
            out.append(("req", cur))
            cur = None
        elif ln.startswith("MODE"):
            out.append(("mode", ln))
        elif ln.startswith("AUDIO"):
            out.append(("audio", ln))
    return out


def test_serve_protocol_matches_the_restated_requests():
    assert BIN.exists(), "g4_serve is built by __graft_entry__.build()"
    a = make_prompt(51, 260, vocab=SMALL["vocab"])
    b = make_prompt(52, 180, vocab=SMALL["vocab"])
    reqs = [(0, [2]), (20, list(a)), (16, list(a[:200]) + list(b[:30])), ("BENCH_MODE 2 0", None), (20, list(b)),
            ("BENCH_MODE 2 1", None), ("AUDIO_RESET", None)]
    lines = []
    for r, p in reqs:
        lines.append(r if p is None else f"{r} " + " ".join(map(str, p)))
    proc = subprocess.run([str(BIN), "ckpt", "index", "/dev/null", "0"], input="\n".join(lines) + "\n", text=True,
                          capture_output=True, env=_env(), timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    got = _parse(proc.stdout.splitlines())
    ref = OracleConversations(dict(SMALL), 1, 32)
    try:
        it = iter(got)
        for r, p in reqs:
            kind, body = next(it)
            if p is None:
                if r == "BENCH_MODE 2 0":
                    assert body == "MODE k=2 tree=0"
                    ref.set_k(2)
                elif r == "BENCH_MODE 2 1":
                    assert body == "MODE_ERROR"
                else:
                    assert body == "AUDIO_UNSUPPORTED"
                continue
            assert kind == "req"
            want, start, _ = ref.request(p, r)
            assert body["gen"] == want
            assert int(body["timing"]["reused"]) == start and int(body["timing"]["prompt"]) == len(p)
            if r > 0:
                assert [body["first"]] + body["tok"] == want  # the streamed tokens are the GEN tokens
                assert int(body["timing"]["decode_tokens"]) == len(want) - 1
    finally:
        ref.close()
    # the third request shares 200 tokens with the second one's conversation
    assert int(got[2][1]["timing"]["reused"]) == 200
