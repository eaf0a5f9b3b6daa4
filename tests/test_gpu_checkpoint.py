"""Engines loaded from checkpoints in the reference's format (g4_engine_create_from_checkpoint)
against the oracle holding the same weights: the checkpoint is written from the oracle's model
(another seed than the engine's default, two layers with a layer_scalar other than 1, weights as
I32 or U8 weight_packed, read through the header or the reference's index file), and the
engine's greedy tokens, drafting trace and hidden states must equal the oracle's.  A checkpoint of
the default synthetic weights gives the generated engine's tokens."""
import numpy as np
import pytest

from oracle_lib import OracleModel, e2e_config, make_prompt

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402
from test_checkpoint import make_index  # noqa: E402

SMALL = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024)


@pytest.fixture(scope="module")
def scaled(tmp_path_factory):
    d = tmp_path_factory.mktemp("gck")
    m = OracleModel(e2e_config(**SMALL, seed=4242))
    m.set_layer_scalar(1, 0.5)
    m.set_layer_scalar(3, 1.25)
    m.write_checkpoint(d / "model.safetensors")
    m.write_checkpoint(d / "u8.safetensors", packed_u8=True)
    make_index(d / "model.safetensors", d / "index.tsv")
    yield d, m
    m.close()


@pytest.mark.parametrize("form", ["header", "index", "u8"])
def test_checkpoint_engine_matches_oracle(scaled, form):
    d, om = scaled
    ck = {"header": lambda: g4.Checkpoint(d),
          "index": lambda: g4.Checkpoint(d / "model.safetensors", d / "index.tsv"),
          "u8": lambda: g4.Checkpoint(d / "u8.safetensors")}[form]()
    eng = g4.Engine(g4.engine_config(seed=4242, ctx_max=1024), checkpoint=ck)
    ck.close()  # the engine holds its own copy of the weights
    try:
        assert (eng.cfg.hidden, eng.cfg.n_layers, eng.cfg.mlp, eng.cfg.vocab) == (512, 5, 1024, 4096)
        toks = make_prompt(5, 8, vocab=4096)
        G_g, h_g = eng.forward(toks, 0)
        G_o, h_o = om.forward(toks, 0)
        assert list(G_g) == list(G_o)
        assert np.array_equal(h_g, h_o)
        p = make_prompt(6, 300, vocab=4096)
        t_g, s_g = eng.generate(p, 48)
        t_o, s_o, tr_o = om.generate(p, 48, trace=True)
        assert list(t_g) == list(t_o)
        assert s_g["rounds"] == s_o["rounds"] and s_g["accepted"] == s_o["accepted"]
        assert np.array_equal(eng.trace(), tr_o)
        assert g4.device_status() == 0
    finally:
        eng.close()


def test_layer_scalars_change_the_model(scaled):
    """The scalars are read: the same weights with every scalar 1 give other hidden states."""
    d, om = scaled
    plain = OracleModel(e2e_config(**SMALL, seed=4242))
    try:
        toks = make_prompt(5, 8, vocab=4096)
        _, h1 = plain.forward(toks, 0)
        _, h2 = om.forward(toks, 0)
        assert not np.array_equal(h1, h2)
    finally:
        plain.close()


def test_checkpoint_of_default_weights_gives_the_generated_engine(tmp_path):
    cfg = dict(SMALL)
    om = OracleModel(e2e_config(**cfg))
    om.write_checkpoint(tmp_path / "model.safetensors")
    om.close()
    ck = g4.Checkpoint(tmp_path)
    a = g4.Engine(g4.engine_config(ctx_max=1024), checkpoint=ck)
    ck.close()
    b = g4.Engine(g4.engine_config(**cfg))
    try:
        p = make_prompt(7, 260, vocab=4096)
        ta, _ = a.generate(p, 40)
        tb, _ = b.generate(p, 40)
        assert list(ta) == list(tb)
    finally:
        a.close()
        b.close()


def test_serve_loads_the_reference_arguments(scaled):
    """g4_serve <ckpt> <index> <prompt> <n_new>, the reference's positional arguments: the
    checkpoint directory and its index are loaded; the GEN tokens are the oracle's."""
    import os
    import pathlib
    import subprocess
    d, om = scaled
    binary = pathlib.Path(g4.LIB_PATH).parent / "g4_serve"
    p = make_prompt(8, 200, vocab=4096)
    env = dict(os.environ, ENGINE_SERVE="1", ENGINE_CTX="1024", G4_SEED="4242")
    proc = subprocess.run([str(binary), str(d), str(d / "index.tsv"), "/dev/null", "0"],
                          input="24 " + " ".join(map(str, p)) + "\n", text=True, capture_output=True, env=env,
                          timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert "checkpoint model hidden=512 layers=5" in proc.stderr
    gen = next(ln for ln in proc.stdout.splitlines() if ln.startswith("GEN:"))
    got = [int(x) for x in gen.split()[1:]]
    want = [om.prefill(p)]
    toks, _ = om.decode(1 << 30, 23)
    want += [int(t) for t in toks]
    for i, t in enumerate(want):
        if t in (1, 106):
            want = want[: i + 1]
            break
    assert got == want
