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
half a minute per prompt on eight cores; the two prompts that those variants change are checked."""
import pathlib
import sys

import numpy as np
import pytest

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import make_golden_e2b as golden  # noqa: E402

FIXTURE = HERE / "golden" / "e2e_e2b_ref.npz"
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
