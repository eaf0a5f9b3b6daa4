"""The oracle on the reference's own model shape against the reference engine's own tokens.

The reference engine (engine/gemma4_engine.cpp) hard-codes the Gemma-4 E2B architecture: 35
layers, every fifth global with 512-wide heads and proportional RoPE, KV sharing from layer 15 on
with a double-wide MLP there, per-layer embeddings and layer scalars.  tests/golden/e2e_e2b_ref.npz
holds the greedy tokens that the reference engine binary, compiled from its sources, produced on a
checkpoint of the oracle's seeded E2B-shaped model (tests/golden/make_golden_e2b.py: four prompts of
100 tokens, eight new tokens each, four layer scalars other than 1).  Here the plain-C oracle,
without any of the reference's kernels, must produce the same tokens; the script that made the
fixture also showed that the same model without its per-layer embeddings, or with every layer
scalar 1, gives other first tokens on two of the four prompts.  Needs about 8 GB of host memory and
half a minute per prompt on eight cores; the two prompts that those variants change are checked.

tests/golden/e2e_e2b_spec_ref.npz holds the same engine's speculative rounds with prompt lookup as
the drafter (the MTP drafter capped at 0 steps): 220-token prompts, so that every verify pass of 2-4
rows runs the split-KV attention, 24 new tokens, and the engine's ngram_rounds / rounds counts, in
both decode modes (int8 verify passes and ENGINE_DECODE_INT8=0).  One of its prompts is checked
here in each mode, tokens and counts.  tests/golden/e2e_e2b_serve_ref.npz holds a session of the
engine as a server through its prefix cache, checked request by request, and
tests/golden/e2e_e2b_fake_ref.npz speculative rounds after ENGINE_FAKE_CTX=600 seeded positions."""
import pathlib
import sys

import numpy as np
import pytest

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import make_golden_e2b as golden  # noqa: E402

FIXTURE = HERE / "golden" / "e2e_e2b_ref.npz"
SPEC_FIXTURE = HERE / "golden" / "e2e_e2b_spec_ref.npz"
SPEC_CHECKED = 2  # its lookups are rejected once before the model settles
SERVE_FIXTURE = HERE / "golden" / "e2e_e2b_serve_ref.npz"
FAKE_FIXTURE = HERE / "golden" / "e2e_e2b_fake_ref.npz"
CHECKED = (1, 2)  # the prompts whose first token moves without per-layer embeddings or scalars


@pytest.fixture(scope="module")
def fixture():
    g = np.load(FIXTURE)
    assert int(g["seed"]) == golden.SEED and int(g["n_new"]) == golden.N_NEW
    assert dict(zip(g["scalar_layers"].tolist(), g["scalar_values"].tolist())) == golden.SCALARS
    return g


def test_fixture_prompts_are_the_scripts(fixture):
    """The stored prompts are the generator's, so the fixture and the script describe one case."""
    for i, p in enumerate(golden.prompts()):
        assert np.array_equal(fixture["prompts"][i], p)


def test_oracle_matches_the_reference_engine_on_e2b(fixture):
    m = golden.e2b_oracle()
    try:
        for i in CHECKED:
            want = [int(t) for t in fixture["tokens"][i] if t >= 0]
            got = [int(t) for t in m.generate(fixture["prompts"][i], golden.N_NEW)[0]]
            assert got == want, f"prompt {i}"
    finally:
        m.close()


@pytest.mark.parametrize("dec", [1, 0], ids=["int8", "decode_int8_0"])
def test_oracle_matches_the_reference_engine_speculative(dec):
    """dec 0 is ENGINE_DECODE_INT8=0 (gemma4_engine.cpp:1600): float verify passes.  On this prompt the
    two modes give different tokens, and the oracle follows the engine in both."""
    g = np.load(SPEC_FIXTURE)
    sfx = "" if dec else "_dec0"
    assert int(g["seed"]) == golden.SEED and int(g["n_new"]) == golden.SPEC_NEW
    assert not np.array_equal(g["tokens"][SPEC_CHECKED], g["tokens_dec0"][SPEC_CHECKED])
    p = golden.spec_prompts()[SPEC_CHECKED]
    assert np.array_equal(g["prompts"][SPEC_CHECKED], p)
    m = golden.e2b_oracle(decode_int8=dec, **golden.SPEC)
    try:
        toks, st = m.generate(p, golden.SPEC_NEW)
        assert [int(t) for t in toks] == [int(t) for t in g["tokens" + sfx][SPEC_CHECKED] if t >= 0]
        assert (st["ngram_rounds"], st["rounds"]) == (int(g["ngram_rounds" + sfx][SPEC_CHECKED]),
                                                      int(g["rounds" + sfx][SPEC_CHECKED]))
        assert st["ngram_rounds"] > 0 and st["accepted"] > 0  # lookups were drafted and accepted
    finally:
        m.close()


def test_prefix_cache_slots_match_the_reference_engine_serving():
    """tests/golden/e2e_e2b_serve_ref.npz: the engine as a server (ENGINE_SERVE=1) with three
    conversation slots: continuation, switch, eviction and repeat.  OracleConversations, the
    restated slot policy that the GPU request tests hold the CUDA engine to, gives the same tokens,
    reused positions and slots for every request."""
    from oracle_lib import OracleConversations
    g = np.load(SERVE_FIXTURE)
    assert int(g["seed"]) == golden.SEED and int(g["slots"]) == golden.SERVE_SLOTS
    reqs = golden.serve_requests()
    for i, p in enumerate(reqs):
        assert np.array_equal(g["requests"][i][: len(p)], p) and (g["requests"][i][len(p):] == -1).all()
    assert sorted(set(g["slot"].tolist())) == [0, 1, 2] and (g["reused"] > 0).sum() >= 3
    conv = OracleConversations(golden.e2b_oracle, golden.SERVE_SLOTS, int(g["min_reuse"]))
    try:
        for i, p in enumerate(reqs):
            toks, start, slot = conv.request(p, int(g["n_new"]))
            assert toks == [int(t) for t in g["tokens"][i] if t >= 0], i
            assert (start, slot) == (int(g["reused"][i]), int(g["slot"][i])), i
    finally:
        conv.close()


def test_fake_context_matches_the_reference_engine():
    """tests/golden/e2e_e2b_fake_ref.npz: ENGINE_FAKE_CTX=600 (the engine's seeded K/V rows before the
    prompt, gemma4_engine.cpp:1249-1250) and speculative rounds with prompt lookup; the oracle's
    fake_ctx and decode give the engine's tokens and round counts."""
    g = np.load(FAKE_FIXTURE)
    assert int(g["seed"]) == golden.SEED and int(g["fake_n"]) == golden.FAKE_N
    i = 1  # its tokens change three times
    p = golden.fake_prompts()[i]
    assert np.array_equal(g["prompts"][i], p)
    m = golden.e2b_oracle(**golden.SPEC)
    try:
        m.fake_ctx(golden.FAKE_N)
        toks, st = m.generate(p, int(g["n_new"]))
        assert [int(t) for t in toks] == [int(t) for t in g["tokens"][i] if t >= 0]
        assert (st["ngram_rounds"], st["rounds"]) == (int(g["ngram_rounds"][i]), int(g["rounds"][i]))
    finally:
        m.close()


def test_the_comparison_can_fail(fixture):
    """Without its per-layer embeddings the same model gives another first token on a checked
    prompt, so agreement above is not a property of every model of this shape."""
    i = CHECKED[0]
    m = golden.e2b_oracle(ple=0)
    try:
        assert int(m.generate(fixture["prompts"][i], 1)[0][0]) != int(fixture["tokens"][i][0])
    finally:
        m.close()


def test_oracle_matches_the_reference_engine_on_the_float_path(fixture):
    """ENGINE_PREFILL_INT8=0 and ENGINE_DECODE_INT8=0: the reference runs its fused float tasks for
    the MLP and the per-layer embeddings; the oracle's float linears around the same element-wise
    steps give the engine's tokens, which differ from the int8 path's on this prompt."""
    i = CHECKED[0]
    want = [int(t) for t in fixture["tokens_float"][i] if t >= 0]
    assert want != [int(t) for t in fixture["tokens"][i] if t >= 0]
    m = golden.e2b_oracle(prefill_int8=0, decode_int8=0)
    try:
        assert [int(t) for t in m.generate(fixture["prompts"][i], golden.N_NEW)[0]] == want
    finally:
        m.close()
