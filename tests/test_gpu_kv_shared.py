"""KV sharing (owner_of, gemma4_engine.cpp:1251; the E2B model's last 20 layers): layers from
kv_owners on have a q projection only and read the K/V cache of the last owner of their type.  The
engine against the oracle with the same sharing, 10 layers of which 5 shared (sliding layers 5-8
read layer 3's cache, global layer 9 reads layer 4's): hidden states of a prefill block, tokens and
per-round trace of prompt lookup and MTP rounds (the drafter reads the target's last sliding and
global caches through the same mapping), int8 and float verify passes, graphs and eager rounds, the
tensor-core prefill, the fake context (filled over the owners only), and a checkpoint whose shared
layers carry no k/v projections.  With mlp_shared the shared layers' MLP is twice as wide (the E2B
model's 12,288 against 6,144)."""
import numpy as np
import pytest

from oracle_lib import OracleModel, e2e_config, make_prompt

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

SHARED = dict(hidden=512, n_layers=10, mlp=1024, vocab=4096, ctx_max=1024, kv_owners=5)
WIDE = dict(SHARED, mlp_shared=2048)


@pytest.mark.parametrize("cfg", [SHARED, WIDE], ids=["shared", "wide"])
def test_forward_matches_oracle(cfg):
    om = OracleModel(e2e_config(**cfg))
    eng = g4.Engine(g4.engine_config(**cfg))
    try:
        toks = make_prompt(3, 8, vocab=4096)
        G_g, h_g = eng.forward(toks, 0)
        G_o, h_o = om.forward(toks, 0)
        assert list(G_g) == list(G_o)
        assert np.array_equal(h_g, h_o)
    finally:
        eng.close()
        om.close()


@pytest.mark.parametrize("ngram,graphs,decode_int8,prefill_tc,wide", [(2, 1, 1, 1, 0), (0, 1, 1, 1, 0), (0, 0, 1, 0, 0),
                                                                       (2, 1, 0, 1, 0), (0, 2, 1, 3, 0), (2, 1, 1, 1, 1),
                                                                       (0, 0, 0, 0, 1)])
def test_generate_matches_oracle(ngram, graphs, decode_int8, prefill_tc, wide):
    cfg = dict(WIDE if wide else SHARED, ngram=ngram, decode_int8=decode_int8)
    om = OracleModel(e2e_config(**cfg))
    eng = g4.Engine(g4.engine_config(**cfg, graphs=graphs, prefill_tc=prefill_tc))
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


def test_fake_context_over_the_owners():
    om = OracleModel(e2e_config(**SHARED))
    eng = g4.Engine(g4.engine_config(**SHARED))
    try:
        om.fake_ctx(400)
        eng.fake_ctx(400)
        prompt = make_prompt(7, 40, vocab=4096)
        tg, _ = eng.generate(prompt, 24)
        to, _ = om.generate(prompt, 24)
        assert list(tg) == list(to)
    finally:
        eng.close()
        om.close()


def test_shared_checkpoint_matches_oracle(tmp_path):
    om = OracleModel(e2e_config(**dict(WIDE, seed=991)))
    try:
        om.write_checkpoint(tmp_path / "model.safetensors")
        ck = g4.Checkpoint(tmp_path)
        eng = g4.Engine(g4.engine_config(seed=991, ctx_max=1024), checkpoint=ck)
        ck.close()
        try:
            assert (eng.cfg.n_layers, eng.cfg.kv_owners, eng.cfg.mlp, eng.cfg.mlp_shared) == (10, 5, 1024, 2048)
            prompt = make_prompt(8, 260, vocab=4096)
            tg, _ = eng.generate(prompt, 32)
            to, _, tro = om.generate(prompt, 32, trace=True)
            assert list(tg) == list(to)
            assert np.array_equal(eng.trace(), tro)
        finally:
            eng.close()
    finally:
        om.close()


def test_engine_refuses_a_shared_layer_without_an_owner():
    with pytest.raises(RuntimeError, match="no global layer"):
        g4.Engine(g4.engine_config(**dict(SHARED, kv_owners=3)))
