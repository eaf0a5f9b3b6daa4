"""The end-to-end engine on the GPU against the CPU oracle's restatement of the same synthetic
model, drafter and chain-mode speculative loop (oracle/g4_oracle_e2e.c), at reduced dimensions
where the oracle is fast.  Forward passes are compared on the final-normed hidden states (bit for
bit) and the greedy tokens; draft steps on the drafted token and next hidden; generation on the
token sequence.

The only non-bit-exact step on the path is expf in the per-(row, head) attention of the first
64 prompt positions and in the split-KV merge (glibc's expf vs a correctly rounded exp, one ulp
apart in ~6e-4 of arguments); hidden states must therefore match in at least 99.9% of elements,
and every greedy token must match.
"""
import numpy as np
import pytest

from oracle_lib import OracleModel, e2e_config, make_prompt

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

SMALL = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024)


@pytest.fixture(scope="module")
def pair():
    cfg = e2e_config(**SMALL)
    om = OracleModel(cfg)
    eng = g4.Engine(g4.engine_config(**SMALL))
    yield om, eng
    eng.close()
    om.close()


def same_frac(a, b):
    return float(np.mean(np.ascontiguousarray(a, np.float32).view(np.uint32) == np.ascontiguousarray(b, np.float32).view(np.uint32)))


def test_forward_prefill_and_verify_blocks(pair):
    om, eng = pair
    prompt = make_prompt(3, 300, vocab=4096)
    done = 0
    # prefill blocks of 32 (int8 path), covering per-(row, head), tiled and the last partial block
    while done < 300:
        M = min(32, 300 - done)
        last = done + M == 300
        Gg, hg = eng.forward(prompt[done:done + M], done, want=last, hf=M - 1 if last else 0, int8=True)
        Go, ho = om.forward(prompt[done:done + M], done, want=last, hf=M - 1 if last else 0, int8=True)
        if last:
            assert Gg[M - 1] == Go[M - 1]
            assert same_frac(hg[M - 1], ho[M - 1]) >= 0.999
        done += M
    # verify blocks at M = 1..4 past the split-KV threshold, int8 and float paths
    pos = 300
    for M, int8 in [(4, True), (3, True), (2, False), (1, True)]:
        toks = make_prompt(pos + M, M, vocab=4096)
        Gg, hg = eng.forward(toks, pos, want=True, hf=0, int8=int8)
        Go, ho = om.forward(toks, pos, want=True, hf=0, int8=int8)
        assert list(Gg) == list(Go), (M, int8)
        assert same_frac(hg, ho) >= 0.999
        pos += M


def test_draft_steps(pair):
    om, eng = pair
    prompt = make_prompt(4, 260, vocab=4096)
    done = 0
    while done < 260:
        M = min(32, 260 - done)
        eng.forward(prompt[done:done + M], done, want=False, int8=True)
        om.forward(prompt[done:done + M], done, want=False, int8=True)
        done += M
    h = np.ascontiguousarray(np.random.default_rng(0).standard_normal(512).astype(np.float32))
    tok = int(prompt[-1])
    for j in range(3):
        tg, hg = eng.draft(tok, h, 260 + j, 259)
        to, ho = om.draft(tok, h, 260 + j, 259)
        assert tg == to
        assert same_frac(hg, ho) >= 0.999
        tok, h = tg, hg


def test_generate_matches_oracle(pair):
    om, eng = pair
    prompt = make_prompt(5, 320, vocab=4096)
    tg, sg = eng.generate(prompt, 40)
    to, so = om.generate(prompt, 40)
    assert list(tg) == list(to)
    assert sg["rounds"] == so["rounds"] and sg["accepted"] == so["accepted"]


@pytest.mark.parametrize("ngram,graphs", [(0, 1), (0, 0), (2, 0)])
def test_generate_graph_replay_and_eager_agree_with_oracle(ngram, graphs):
    """Decode rounds replayed from captured graphs (positions read on the device) and launched
    eagerly give the oracle's tokens, with MTP drafts (ngram 0) and with prompt lookup."""
    om = OracleModel(e2e_config(**SMALL, ngram=ngram))
    eng = g4.Engine(g4.engine_config(**SMALL, ngram=ngram, graphs=graphs))
    try:
        prompt = make_prompt(6, 300, vocab=4096)
        tg, sg = eng.generate(prompt, 32)
        to, so = om.generate(prompt, 32)
        assert list(tg) == list(to)
        assert sg["rounds"] == so["rounds"] and sg["accepted"] == so["accepted"]
        assert sg["verify_passes"] == sg["rounds"] and sg["verify_rows"] >= sg["rounds"]
        if ngram == 0:
            assert sg["draft_steps"] == 3 * sg["rounds"] and sg["draft_gpu_ms"] > 0
        assert sg["h2d_bytes"] > 0 and sg["d2h_bytes"] > 0
    finally:
        eng.close()
        om.close()


def test_fake_context_generate_matches_oracle():
    """ENGINE_FAKE_CTX: a 600-position LCG context, then a short prompt and decode on top of it."""
    om = OracleModel(e2e_config(**SMALL))
    eng = g4.Engine(g4.engine_config(**SMALL))
    try:
        om.fake_ctx(600)
        eng.fake_ctx(600)
        prompt = make_prompt(7, 40, vocab=4096)
        tg, _ = eng.generate(prompt, 24)
        to, _ = om.generate(prompt, 24)
        assert list(tg) == list(to)
    finally:
        eng.close()
        om.close()


def test_generate_cfg4_golden():
    """configs[4] at full size: the seeded 6,841-token prompt, 256 greedy tokens, against the
    oracle's tokens and round statistics stored by tests/golden/make_golden_e2e.py."""
    import pathlib
    d = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "e2e_cfg4.npz")
    eng = g4.Engine(g4.engine_config())
    try:
        assert eng.cfg.seed == int(d["seed"])
        toks, st = eng.generate(d["prompt"], 256)
        assert list(toks) == list(d["tokens"])
        assert (st["rounds"], st["ngram_rounds"], st["accepted"]) == (int(d["rounds"]), int(d["ngram_rounds"]),
                                                                       int(d["accepted"]))
    finally:
        eng.close()
