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
    to, so, tro = om.generate(prompt, 40, trace=True)
    assert list(tg) == list(to)
    assert sg["rounds"] == so["rounds"] and sg["accepted"] == so["accepted"]
    assert np.array_equal(eng.trace(), tro)


# (ngram, graphs, decode_int8, vocab): MTP drafts (ngram 0) and prompt lookup; rounds replayed as one
# loop graph with conditional nodes (graphs 1), as graphs of single passes launched from the host
# (graphs 2) and eagerly (graphs 0); int8 and float (ENGINE_DECODE_INT8=0) verify passes; a vocab of
# 16,384 gives 128 drafter centroids, so the drafter's top-32 selection is a real choice.
CASES = [(0, 1, 1, 4096), (0, 0, 1, 4096), (2, 0, 1, 4096), (2, 2, 1, 4096), (2, 1, 0, 4096), (2, 0, 0, 4096),
         (0, 1, 0, 4096), (0, 1, 1, 16384), (0, 0, 1, 16384), (2, 1, 1, 16384)]


@pytest.mark.parametrize("ngram,graphs,decode_int8,vocab", CASES)
def test_generate_agrees_with_oracle(ngram, graphs, decode_int8, vocab):
    """Tokens, round counts and the per-round trace (drafts, acceptance) equal the oracle's."""
    cfg = dict(SMALL, vocab=vocab, ngram=ngram, decode_int8=decode_int8)
    om = OracleModel(e2e_config(**cfg))
    eng = g4.Engine(g4.engine_config(**cfg, graphs=graphs))
    try:
        prompt = make_prompt(6, 300, vocab=vocab)
        tg, sg = eng.generate(prompt, 32)
        to, so, tro = om.generate(prompt, 32, trace=True)
        assert list(tg) == list(to)
        assert sg["rounds"] == so["rounds"] and sg["accepted"] == so["accepted"]
        assert sg["ngram_rounds"] == so["ngram_rounds"] and sg["drafted"] == so["drafted"]
        assert np.array_equal(eng.trace(), tro)
        assert sg["verify_passes"] == sg["rounds"] and sg["verify_rows"] >= sg["rounds"]
        if ngram == 0:
            assert sg["draft_steps"] == 3 * sg["rounds"] and sg["draft_gpu_ms"] > 0
        assert sg["d2h_bytes"] > 0 and sg["kernel_launches"] > sg["rounds"]
        assert g4.device_status() == 0
    finally:
        eng.close()
        om.close()


@pytest.mark.parametrize("graphs,lim", [(1, 8), (0, 8), (1, 200)])
def test_screen_backoff_gives_the_same_tokens(graphs, lim):
    """head_screen 2 (the default) skips the certified screen for 1, 2, 4 .. 64 passes after a pass
    whose screen fell back, and runs the full exact head at once.  With a survivor limit of 8 the
    screen falls back on every pass it runs; the tokens, statistics and per-round trace equal the
    oracle's (its pick is over the full exact head) for head_screen 2, 1 (the screen every pass)
    and 0 (the full exact head every pass)."""
    cfg = dict(SMALL, ngram=0, screen_lim=lim)
    om = OracleModel(e2e_config(**cfg))
    engines = {hs: g4.Engine(g4.engine_config(**cfg, head_screen=hs, graphs=graphs)) for hs in (2, 1, 0)}
    try:
        prompt = make_prompt(9, 300, vocab=4096)
        to, so, tro = om.generate(prompt, 40, trace=True)
        for hs, eng in engines.items():
            tg, sg = eng.generate(prompt, 40)
            assert list(tg) == list(to), hs
            assert sg["rounds"] == so["rounds"] and sg["accepted"] == so["accepted"], hs
            assert np.array_equal(eng.trace(), tro), hs
            if hs == 1:
                assert sg["screen_skipped"] == 0
            if hs == 2 and lim == 8:
                assert sg["head_fallbacks"] == sg["verify_passes"]  # every pass read the full head
                # screened passes: 1 + the probes after back-offs of 1, 2, 4, ... passes
                assert sg["screen_skipped"] >= sg["verify_passes"] - 8 and sg["screen_skipped"] > 0
        assert g4.device_status() == 0
    finally:
        for eng in engines.values():
            eng.close()
        om.close()


def test_decode_calls_resume_and_export_state():
    """Decode in several calls (each one loop-graph launch) continues the same token stream as one
    call, and the exported history is the prompt plus every committed token."""
    cfg = dict(SMALL, ngram=0)
    a = g4.Engine(g4.engine_config(**cfg))
    b = g4.Engine(g4.engine_config(**cfg))
    try:
        prompt = make_prompt(8, 280, vocab=4096)
        ta, _ = a.generate(prompt, 25)
        first = b.prefill(prompt)
        got = [first]
        for _ in range(6):
            out = np.zeros(64, np.int32)
            n, _ = b.decode(2, 64, out)  # two rounds per call, every committed token returned
            got += list(out[:n])
        k = min(len(got), len(ta))
        assert k >= 13 and got[:k] == list(ta[:k])
        _, _, seq, h, P = b.export_state(0, kv=False)
        assert list(seq[:280]) == list(prompt) and seq.size >= 281
        assert P == seq.size - 2  # the last committed token is verified at the next round's first row
        assert list(seq[280:280 + len(got)]) == got[: seq.size - 280]
    finally:
        a.close()
        b.close()


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


@pytest.mark.parametrize("name", ["e2e_cfg4", "e2e_cfg4_float", "e2e_cfg4_ngram0"])
def test_generate_cfg4_golden(name):
    """configs[4] at full size: the seeded 6,841-token prompt, 256 greedy tokens, against the
    oracle's tokens, round statistics and per-round trace stored by tests/golden/make_golden_e2e.py:
    the default engine (int8 verify passes, prompt lookup), ENGINE_DECODE_INT8=0 (float verify
    passes, whose tokens must be bit-exact), and prompt lookup off (every round drafts 3 tokens with
    the full-size MTP drafter, top 32 of 2,048 centroids, and verifies 4 rows)."""
    import pathlib
    path = pathlib.Path(__file__).resolve().parent / "golden" / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"{path.name} not generated")
    d = np.load(path)
    kw = {}
    if "decode_int8" in d:
        kw = dict(decode_int8=int(d["decode_int8"]), ngram=int(d["ngram"]))
    eng = g4.Engine(g4.engine_config(**kw))
    try:
        assert eng.cfg.seed == int(d["seed"])
        toks, st = eng.generate(d["prompt"], 256)
        assert list(toks) == list(d["tokens"])
        assert (st["rounds"], st["ngram_rounds"], st["accepted"]) == (int(d["rounds"]), int(d["ngram_rounds"]),
                                                                       int(d["accepted"]))
        if "trace" in d:
            assert np.array_equal(eng.trace(), d["trace"])
    finally:
        eng.close()


def test_fused_segments_match_per_kernel_path():
    """At the full width (hidden 2048, MLP 8192, 30 layers), verify passes of M = 2..4 rows through
    the persistent segment kernels give the same greedy tokens and final hidden states, bit for bit,
    as the one-kernel-per-step path, and the same as the oracle."""
    cfg = dict(ctx_max=1024)
    a = g4.Engine(g4.engine_config(**cfg, fused_layers=1))
    b = g4.Engine(g4.engine_config(**cfg, fused_layers=0))
    om = OracleModel(e2e_config(**cfg))
    try:
        prompt = make_prompt(9, 260)
        for eng in (a, b):
            done = 0
            while done < 260:
                M = min(32, 260 - done)
                eng.forward(prompt[done:done + M], done, want=False, int8=True)
                done += M
        done = 0
        while done < 260:
            M = min(32, 260 - done)
            om.forward(prompt[done:done + M], done, want=False, int8=True)
            done += M
        pos = 260
        for M in (4, 2, 3):
            toks = make_prompt(pos + M, M)
            Ga, ha = a.forward(toks, pos, want=True, hf=0, int8=True)
            Gb, hb = b.forward(toks, pos, want=True, hf=0, int8=True)
            Go, ho = om.forward(toks, pos, want=True, hf=0, int8=True)
            assert np.array_equal(ha.view(np.uint32), hb.view(np.uint32)), M
            assert list(Ga) == list(Gb) == list(Go), M
            assert same_frac(ha, ho) >= 0.999
            pos += M
        assert g4.device_status() == 0
    finally:
        a.close()
        b.close()
        om.close()


@pytest.mark.parametrize("cfg", [dict(SMALL), dict(ctx_max=2048), dict(SMALL, prefill_block=7)])
def test_tensor_core_prefill_matches_block_prefill(cfg):
    """The prompt's full blocks prefilled at once with the tensor-core W4A8 GEMM write the same KV
    cache, hidden state and first token, bit for bit, as prefill block by block through the GEMV
    path; at the full width and at reduced dimensions; with the attention taking one row of a head
    per block (prefill_tc 1) or four (3).  Prefill blocks of 7 rows put the switch from the per-row
    to the tiled attention variant (the first block ending past position 64) inside a group of four
    rows, which then runs row by row."""
    vocab = cfg.get("vocab", 262144)
    prompt = make_prompt(11, 777, vocab=vocab)
    outs = []
    for tc in (1, 3, 0):
        eng = g4.Engine(g4.engine_config(**cfg, prefill_tc=tc))
        try:
            first = eng.prefill(prompt)
            K, V, seq, h, P = eng.export_state(777)
            outs.append((first, K, V, h, P))
        finally:
            eng.close()
    f0, K0, V0, h0, P0 = outs[-1]
    for f1, K1, V1, h1, P1 in outs[:-1]:
        assert f1 == f0 and P1 == P0
        assert np.array_equal(K1, K0) and np.array_equal(V1, V0)
        assert np.array_equal(h1.view(np.uint32), h0.view(np.uint32))


def test_shared_weight_streams_decode_concurrently():
    """Independent request streams: engines over one engine's weights, each with its own prompt, KV
    cache and stream, decoding at the same time (asynchronous calls), commit the same tokens as the
    oracle's run of each prompt alone."""
    cfg = dict(SMALL, ngram=0)
    base = g4.Engine(g4.engine_config(**cfg))
    streams = [base] + [g4.Engine(g4.engine_config(**cfg), share=base) for _ in range(3)]
    om = OracleModel(e2e_config(**cfg))
    try:
        prompts = [make_prompt(20 + i, 250 + 7 * i, vocab=4096) for i in range(4)]
        firsts = [eng.prefill(p) for eng, p in zip(streams, prompts)]
        start = torch.cuda.Event(enable_timing=True)
        start.record()
        for eng in streams:
            eng.decode_async(6, 1 << 20, start)
        got = [eng.decode_wait(start) for eng in streams]
        for p, f, (toks, st, ms) in zip(prompts, firsts, got):
            ref, _ = om.generate(p, 1 + len(toks))
            assert [f] + list(toks) == list(ref[: 1 + len(toks)])
            assert st["rounds"] == 6 and ms is not None and ms > 0
        assert g4.device_status() == 0
    finally:
        for eng in streams[1:]:
            eng.close()
        base.close()
        om.close()


def test_copied_stream_decodes_in_the_engine_mode():
    """A stream engine whose first call is an asynchronous decode (its state copied from another
    engine, never prefilled itself) records its round graphs in the engine's decode mode (W4A8 here):
    the same tokens, history and final hidden state as the source engine decoding the same rounds
    (the hidden state tells the int8 verify passes from float ones even where the tokens agree)."""
    cfg = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024)
    a = g4.Engine(g4.engine_config(**cfg))
    b = g4.Engine(g4.engine_config(**cfg), share=a)
    try:
        a.prefill(make_prompt(9, 300, vocab=4096))  # past att_par: the decode runs as graphs
        b.copy_state_from(a)
        out = np.zeros(64, np.int32)
        n, _ = a.decode(8, 64, out)
        b.decode_async(8, 64)
        tb, _, _ = b.decode_wait()
        assert list(out[:n]) == list(tb)
        _, _, seq_a, h_a, P_a = a.export_state(0, kv=False)
        _, _, seq_b, h_b, P_b = b.export_state(0, kv=False)
        assert P_a == P_b and np.array_equal(seq_a, seq_b)
        assert np.array_equal(h_a, h_b)
    finally:
        b.close()
        a.close()
