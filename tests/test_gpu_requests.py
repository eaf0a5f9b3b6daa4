"""Requests through the prefix cache (g4_engine_request: run_req and its conversation slots,
gemma4_engine.cpp:1569-1613) against the same policy restated here over oracle models, one model
per conversation (each holds its own K/V and history, as a slot does): the longest shared prefix
picks the conversation, a stored one that shares more is switched in, a prompt that shares fewer
than slot_min_reuse tokens with every conversation evicts the least recently used slot, and the
prefill starts at min(shared, n - 1).  Tokens, reused positions and the slot used must equal the
restatement's for every request."""
import numpy as np
import pytest

from oracle_lib import OracleModel, e2e_config, make_prompt

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

SMALL = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024)
STOP = (1, 106)


class OracleConversations:
    """run_req's prefix cache over oracle models: [model, keys, kv_len, stamp] per conversation."""

    def __init__(self, cfg, slots, min_reuse):
        self.min_reuse = min_reuse
        self.active = [OracleModel(e2e_config(**cfg)), [], 0, 0]
        self.stored = [[OracleModel(e2e_config(**cfg)), [], 0, 0] for _ in range(slots - 1)]
        self.tick = 0

    def close(self):
        for c in [self.active] + self.stored:
            c[0].close()

    def set_k(self, k):
        for c in [self.active] + self.stored:
            c[0].set_k(k)

    @staticmethod
    def _lcp(keys, kv_len, prompt):
        c = 0
        while c < kv_len and c < len(prompt) and c < len(keys) and keys[c] == prompt[c]:
            c += 1
        return c

    def _swap(self, i):
        self.active, self.stored[i] = self.stored[i], self.active

    def request(self, prompt, max_new):
        prompt = [int(t) for t in prompt]
        n = len(prompt)
        common = self._lcp(self.active[1], self.active[2], prompt)
        self.tick += 1
        slot = 0
        if self.stored:
            best, bc = -1, common
            for i, s in enumerate(self.stored):
                c = self._lcp(s[1], s[2], prompt)
                if c > bc:
                    bc, best = c, i
            if best >= 0:
                self.active[3] = self.tick
                self._swap(best)
                slot, common = best + 1, bc
            elif bc < self.min_reuse:
                v = min(range(len(self.stored)), key=lambda i: self.stored[i][3])  # the first oldest
                self.active[3] = self.tick
                self._swap(v)
                self.active[1], self.active[2] = [], 0
                slot, common = v + 1, 0
            self.active[3] = self.tick
        start = min(common, n - 1)
        m = self.active[0]
        first = m.prefill(prompt, start)
        if max_new <= 0:  # prefill only: the prompt is the conversation
            self.active[1], self.active[2] = prompt, n
            return [], start, slot
        out = [first]
        if max_new > 1 and out[0] not in STOP:
            toks, _ = m.decode(1 << 30, max_new - 1)
            out += [int(t) for t in toks]
        for i, t in enumerate(out):
            if t in STOP:
                out = out[: i + 1]
                break
        seq, P = m.history()
        self.active[1] = [int(t) for t in seq[: P + 1]]
        self.active[2] = min(P + 1, len(self.active[1]))
        return out, start, slot


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
    ref = OracleConversations(cfg, slots, 32)
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
