"""Requests through the prefix cache (g4_engine_request: run_req and its conversation slots,
gemma4_engine.cpp:1569-1613) against the same policy restated over oracle models
(oracle_lib.OracleConversations, itself pinned to the reference engine's serve mode on the E2B
shape), one model per conversation (each holds its own K/V and history, as a slot does): the
longest shared prefix picks the conversation, a stored one that shares more is switched in, a
prompt that shares fewer than slot_min_reuse tokens with every conversation evicts the least
recently used slot, and the prefill starts at min(shared, n - 1).  Tokens, reused positions and the slot used must equal the
restatement's for every request."""
import numpy as np
import pytest

from oracle_lib import OracleConversations, OracleModel, e2e_config, make_prompt

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

SMALL = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024)


def _prompts():
    a = make_prompt(31, 300, vocab=4096)
    b = make_prompt(32, 200, vocab=4096)
    c = make_prompt(33, 150, vocab=4096)
    extra = make_prompt(34, 120, vocab=4096)
    return [
        a,                                        # a new conversation
        np.concatenate([a[:250], extra[:40]]),    # shares 250 tokens with it
        b,                                        # shares nothing: a slot takes the active one
        np.concatenate([a[:200], extra[40:90]]),  # back to the first conversation
        c,
        np.concatenate([b[:180], extra[90:120]]),
        np.concatenate([a[:20], extra[:60]]),     # shares fewer than slot_min_reuse tokens
    ]


@pytest.mark.parametrize("slots", [3, 1])
def test_requests_with_prefix_cache_match_the_restated_policy(slots):
    cfg = dict(SMALL)
    eng = g4.Engine(g4.engine_config(**cfg, slots=slots, slot_min_reuse=32))
    ref = OracleConversations(lambda: OracleModel(e2e_config(**cfg)), slots, 32)
    try:
        reused_any = False
        for i, p in enumerate(_prompts()):
            toks, info = eng.request(p, 24)
            want, start, slot = ref.request(p, 24)
            assert list(toks) == want, i
            assert info["reused"] == start and info["slot"] == slot, (i, info, start, slot)
            assert info["prompt_tokens"] == len(p) and info["tokens"] == len(want)
            reused_any = reused_any or start > 0
        assert reused_any
        assert g4.device_status() == 0
    finally:
        eng.close()
        ref.close()


def test_prefill_from_keeps_the_prefix():
    """g4_engine_prefill_from on a cache that holds the prompt's prefix: the same first token and
    the same decoded tokens as the oracle's prefill from the same position on the same prefix."""
    cfg = dict(SMALL)
    eng = g4.Engine(g4.engine_config(**cfg))
    om = OracleModel(e2e_config(**cfg))
    try:
        a = make_prompt(41, 260, vocab=4096)
        b = np.concatenate([a[:200], make_prompt(42, 77, vocab=4096)])
        assert eng.prefill(a) == om.prefill(a)
        for start in (200, 150, 1):
            f_g = eng.prefill(b, start=start)
            f_o = om.prefill(b, start=start)
            assert f_g == f_o, start
            out = np.zeros(8, np.int32)
            n, _ = eng.decode(4, 8, out)
            want, _ = om.decode(4, 8)
            assert list(out[:n]) == list(want), start
            eng.prefill(b, start=0)
            om.prefill(b, start=0)
    finally:
        eng.close()
        om.close()
