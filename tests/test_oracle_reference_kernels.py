"""The oracle's end-to-end restatement against itself with the reference's own compiled kernels
(oracle/_ref/libg4ref.so: the AVX2 lin_task / i8_task linears, attn_task + attn_merge, attn_tile
and head_task, driven by the reference's thread pool) in place of its C linears, attention and
head, for the synthetic model and for the E2B structures the engine adds: KV sharing (owner_of,
gemma4_engine.cpp:1251), the double-wide MLP of the shared layers, and the per-layer embeddings
(whose three extra linears per layer run through the reference's kernels too).  Hidden states of a
prefill block and greedy tokens of a decode must be bit-identical.  Host only; skipped where the
reference kernels were not built (the reference tree is needed at build time)."""
import numpy as np
import pytest

from oracle_lib import OracleModel, e2e_config, make_prompt, reference

BASE = dict(hidden=512, mlp=1024, vocab=4096, ctx_max=1024)
CASES = {"plain": dict(n_layers=5), "kv_shared_wide": dict(n_layers=10, kv_owners=5, mlp_shared=2048),
         "ple": dict(n_layers=5, ple=1), "e2b_like": dict(n_layers=10, kv_owners=5, mlp_shared=2048, ple=1)}


@pytest.mark.skipif(reference() is None, reason="oracle/_ref/libg4ref.so not built")
@pytest.mark.parametrize("name", list(CASES))
def test_restatement_equals_reference_kernels(name):
    cfg = dict(BASE, **CASES[name])
    a = OracleModel(e2e_config(**cfg))
    b = OracleModel(e2e_config(**cfg))
    try:
        assert b.use_reference_kernels()
        toks = make_prompt(3, 8, vocab=4096)
        ga, ha = a.forward(toks, 0)
        gb, hb = b.forward(toks, 0)
        assert list(ga) == list(gb)
        assert np.array_equal(ha, hb)
        prompt = make_prompt(6, 300, vocab=4096)
        ta, sa = a.generate(prompt, 24)
        tb, sb = b.generate(prompt, 24)
        assert list(ta) == list(tb) and sa == sb
    finally:
        a.close()
        b.close()
