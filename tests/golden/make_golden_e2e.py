"""Generate tests/golden/e2e_cfg4.npz: the configs[4] workload through the CPU end-to-end oracle
(oracle/g4_oracle_e2e.c) — the seeded 6,841-token prompt and the 256 greedily decoded tokens of
the synthetic E2B model with its MTP drafter and prompt lookup.

    python tests/golden/make_golden_e2e.py        (about ten minutes on 8 cores)

The GPU test tests/test_gpu_engine.py::test_generate_cfg4_golden decodes the same prompt on the
engine and compares the tokens.
"""
import pathlib
import sys
import time

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from oracle_lib import OracleModel, e2e_config, make_prompt  # noqa: E402

PROMPT_SEED, N_PROMPT, N_NEW = 4, 6841, 256


def main():
    cfg = e2e_config()
    prompt = make_prompt(PROMPT_SEED, N_PROMPT)
    t0 = time.time()
    m = OracleModel(cfg)
    t1 = time.time()
    toks, st = m.generate(prompt, N_NEW)
    t2 = time.time()
    m.close()
    np.savez_compressed(HERE / "e2e_cfg4.npz", prompt=prompt, tokens=toks, seed=np.uint64(cfg.seed),
                        rounds=st["rounds"], ngram_rounds=st["ngram_rounds"], drafted=st["drafted"],
                        accepted=st["accepted"])
    print(f"create {t1 - t0:.1f}s generate {t2 - t1:.1f}s tokens {len(toks)} stats {st}")
    print(list(toks[:32]))


if __name__ == "__main__":
    main()
