"""Generate the configs[4] end-to-end goldens through the CPU end-to-end oracle
(oracle/g4_oracle_e2e.c): the seeded 6,841-token prompt and the 256 greedily decoded tokens of the
synthetic E2B model with its MTP drafter, plus the per-round trace (drafts, acceptance).

    python tests/golden/make_golden_e2e.py [int8|float|ngram0 ...]   (about ten minutes each on 8 cores)

  int8    e2e_cfg4.npz         the default engine configuration (ENGINE_DECODE_INT8=1, prompt lookup on)
  float   e2e_cfg4_float.npz   ENGINE_DECODE_INT8=0: the verify passes run the float W4G32 path
  ngram0  e2e_cfg4_ngram0.npz  prompt lookup off: every round drafts k = 3 tokens with the MTP drafter
                               and verifies M = 4 rows

tests/test_gpu_engine.py decodes the same prompts on the engine and compares tokens, round counts
and the per-round trace.
"""
import pathlib
import sys
import time

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from oracle_lib import OracleModel, e2e_config, make_prompt  # noqa: E402

PROMPT_SEED, N_PROMPT, N_NEW = 4, 6841, 256
VARIANTS = {"int8": ("e2e_cfg4.npz", {}), "float": ("e2e_cfg4_float.npz", {"decode_int8": 0}),
            "ngram0": ("e2e_cfg4_ngram0.npz", {"ngram": 0})}


def make(variant):
    fname, kw = VARIANTS[variant]
    cfg = e2e_config(**kw)
    prompt = make_prompt(PROMPT_SEED, N_PROMPT)
    t0 = time.time()
    m = OracleModel(cfg)
    t1 = time.time()
    toks, st, trace = m.generate(prompt, N_NEW, trace=True)
    t2 = time.time()
    m.close()
    np.savez_compressed(HERE / fname, prompt=prompt, tokens=toks, seed=np.uint64(cfg.seed), trace=trace,
                        decode_int8=np.int32(cfg.decode_int8), ngram=np.int32(cfg.ngram), rounds=st["rounds"],
                        ngram_rounds=st["ngram_rounds"], drafted=st["drafted"], accepted=st["accepted"])
    print(f"{variant}: create {t1 - t0:.1f}s generate {t2 - t1:.1f}s tokens {len(toks)} stats {st}", flush=True)


if __name__ == "__main__":
    for v in sys.argv[1:] or list(VARIANTS):
        make(v)
