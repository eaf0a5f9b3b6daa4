"""Golden tokens of the reference engine itself on an E2B-shaped synthetic model.

The reference engine (engine/gemma4_engine.cpp) hard-codes the Gemma-4 E2B architecture: hidden
1536, 35 layers (every fifth global, 512-wide heads with proportional RoPE; the others sliding,
256-wide), KV sharing from layer 15 on with a double-wide MLP there (12,288 against 6,144),
per-layer embeddings of 256 per layer, layer scalars, a tied 262,144-token head.  This script
builds that model in the oracle (tests/oracle_lib.py) from a seed, writes it as a checkpoint in the
reference's format (model.safetensors plus the index make_index.py would write), runs the
reference engine binary compiled from its sources (oracle/_ref/gemma4_engine, `make -C oracle
engine`) on it with ENGINE_K=0 (plain greedy decode) and ENGINE_PREFILL_INT8=1 (the int8 branch),
and stores the prompts and the engine's GEN tokens in tests/golden/e2e_e2b_ref.npz (four prompts,
one engine run each, so four first tokens of the full forward).  The oracle's own tokens for the
same model are printed beside them and, as a check that the comparison can fail, the first tokens
of the same model without its per-layer embeddings and with every layer scalar 1.  Needs ~16 GB of
host memory and ~7 GB of temporary disk; run by hand:

    python tests/golden/make_golden_e2b.py
"""
import os
import pathlib
import subprocess
import sys
import tempfile
import time

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE.parent))

from oracle_lib import OracleModel, e2e_config, make_prompt  # noqa: E402
from test_checkpoint import make_index  # noqa: E402

SEED = 20261202
N_PROMPT, N_NEW, N_REQ = 100, 8, 4
# the reference's hard-coded model (gemma4_engine.cpp:1222-1231, ENGINE_SPEC.md dimensions)
E2B = dict(hidden=1536, n_layers=35, mlp=6144, mlp_shared=12288, vocab=262144, kv_owners=15, ple=1, hd_global=512,
           rope_global_quarter=1, drafter=0, k_draft=0, ngram=0, prefill_int8=1, decode_int8=1, ctx_max=1024,
           prefill_block=32, seed=SEED)
SCALARS = {3: 0.75, 14: 1.5, 22: 0.5, 34: 1.25}  # a few layer scalars other than 1 (bf16 values)


def e2b_oracle(scalars=True, **over):
    m = OracleModel(e2e_config(**dict(E2B, **over)))
    if scalars:
        for l, v in SCALARS.items():
            m.set_layer_scalar(l, v)
    return m


def prompts():
    return [make_prompt(SEED % 1000 + i, N_PROMPT) for i in range(N_REQ)]


def main():
    binary = ROOT / "oracle" / "_ref" / "gemma4_engine"
    if not binary.exists():
        sys.exit(f"{binary} missing: make -C oracle engine REF=<reference checkout>")
    ps = prompts()
    t0 = time.time()
    m = e2b_oracle()
    print(f"oracle model built in {time.time() - t0:.0f} s", flush=True)
    with tempfile.TemporaryDirectory() as d:
        d = pathlib.Path(d)
        m.write_checkpoint(d / "model.safetensors")
        make_index(d / "model.safetensors", d / "index.tsv")
        env = dict(os.environ, ENGINE_K="0", ENGINE_PREFILL_INT8="1", ENGINE_CTX="1024",
                   ENGINE_CPUS=",".join(str(i) for i in range(min(8, os.cpu_count() or 1))))
        gens = []
        for i, p in enumerate(ps):  # one run per prompt: each prefill starts at position 0
            (d / "prompt.txt").write_text(" ".join(str(int(t)) for t in p))
            t1 = time.time()
            proc = subprocess.run([str(binary), str(d), str(d / "index.tsv"), str(d / "prompt.txt"), str(N_NEW)],
                                  capture_output=True, text=True, env=env, timeout=3600)
            print(f"reference engine, prompt {i}: {time.time() - t1:.0f} s (rc {proc.returncode})", flush=True)
            if proc.returncode != 0:
                sys.exit(proc.stderr[-3000:])
            gen = next(ln for ln in proc.stdout.splitlines() if ln.startswith("GEN:"))
            gens.append([int(x) for x in gen.split()[1:]])
    m.use_reference_kernels()
    ours = [[int(t) for t in m.generate(p, N_NEW)[0]] for p in ps]
    m.close()
    for g, o in zip(gens, ours):
        print("reference:", g, "\noracle:   ", o)
    for name, over in (("without per-layer embeddings", dict(ple=0)), ("every layer scalar 1", dict(scalars=False))):
        v = e2b_oracle(**over)
        v.use_reference_kernels()
        firsts = [int(v.generate(p, 1)[0][0]) for p in ps]
        v.close()
        print(f"first tokens {name}: {firsts} (reference: {[g[0] for g in gens]})")
    width = max(len(g) for g in gens)
    tok = np.full((N_REQ, width), -1, np.int32)
    for i, g in enumerate(gens):
        tok[i, :len(g)] = g
    np.savez(HERE / "e2e_e2b_ref.npz", prompts=np.stack([np.asarray(p, np.int32) for p in ps]), tokens=tok, seed=SEED,
             n_new=N_NEW, scalar_layers=np.array(list(SCALARS), np.int32),
             scalar_values=np.array(list(SCALARS.values()), np.float32))
    print("agree" if ours == gens else "DIFFER")


if __name__ == "__main__":
    main()
