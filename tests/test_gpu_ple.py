"""Per-layer embeddings (the E2B model's PLE, the int8 branch of gemma4_engine.cpp:1270-1288 and
1379-1388): each token's 256 inputs per layer come from a [vocab][n_layers x 256] table and a
projection of its embedding, and after each layer's MLP a gate of the layer's inputs is projected
back into the residual stream (before the layer scalar).  The engine against the oracle with the
same weights: hidden states of a prefill block, tokens and per-round trace with prompt lookup and
MTP drafts, graphs and eager rounds; and the E2B model's structure at small size (per-layer
embeddings, KV sharing, double-wide MLP in the shared layers)."""
import numpy as np
import pytest

from oracle_lib import OracleModel, e2e_config, make_prompt

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

PLE = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024, ple=1)


def test_forward_matches_oracle():
    om = OracleModel(e2e_config(**PLE))
    eng = g4.Engine(g4.engine_config(**PLE))
    try:
        for toks, pos0 in ((make_prompt(3, 8, vocab=4096), 0), (make_prompt(4, 1, vocab=4096), 8)):
            G_g, h_g = eng.forward(toks, pos0)
            G_o, h_o = om.forward(toks, pos0)
            assert list(G_g) == list(G_o)
            assert np.array_equal(h_g, h_o)
    finally:
        eng.close()
        om.close()


@pytest.mark.parametrize("ngram,graphs", [(2, 1), (0, 1), (2, 0), (0, 2)])
def test_generate_matches_oracle(ngram, graphs):
    cfg = dict(PLE, ngram=ngram)
    om = OracleModel(e2e_config(**cfg))
    eng = g4.Engine(g4.engine_config(**cfg, graphs=graphs))
    try:
        prompt = make_prompt(6, 300, vocab=4096)
        tg, sg = eng.generate(prompt, 32)
        to, so, tro = om.generate(prompt, 32, trace=True)
        assert list(tg) == list(to)
        assert sg["rounds"] == so["rounds"] and sg["accepted"] == so["accepted"]
        assert np.array_equal(eng.trace(), tro)
        assert g4.device_status() == 0
    finally:
        eng.close()
        om.close()


def test_e2b_structure_matches_oracle():
    cfg = dict(PLE, n_layers=10, kv_owners=5, mlp_shared=2048)
    om = OracleModel(e2e_config(**cfg))
    eng = g4.Engine(g4.engine_config(**cfg))
    try:
        toks = make_prompt(3, 8, vocab=4096)
        G_g, h_g = eng.forward(toks, 0)
        G_o, h_o = om.forward(toks, 0)
        assert list(G_g) == list(G_o) and np.array_equal(h_g, h_o)
    finally:
        eng.close()
        om.close()


def test_engine_refuses_ple_with_float_activations():
    with pytest.raises(RuntimeError, match="int8 branch"):
        g4.Engine(g4.engine_config(**dict(PLE, decode_int8=0)))
