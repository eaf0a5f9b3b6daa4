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
of the same model without its per-layer embeddings and with every layer scalar 1.  The same prompts
are also run on the float path (ENGINE_PREFILL_INT8=0, ENGINE_DECODE_INT8=0) into tokens_float.

A second case drives the speculative loop (run_req's draft-verify-accept rounds, :1616-1661) with
prompt lookup as the only drafter: ENGINE_K=3 enters the loop, ENGINE_POLICY=0,0,0 caps the MTP
drafter's steps at 0 (:1621), ENGINE_NGRAM=2 and ENGINE_NGLEN=3 copy up to three tokens after the
latest earlier match of the last two (:1624-1628).  The prompts are 220 tokens long, so every verify
pass of 2-4 rows runs the split-KV attention (M <= 4 past ENGINE_ATT_PAR = 192, :1305).  The engine
loads a drafter checkpoint before it starts; a placeholder with the drafter's tensor names is
written (its values are never read when no draft step runs).  It runs in both decode modes, the
int8 verify passes and ENGINE_DECODE_INT8=0.  The tokens and the engine's ngram_rounds / rounds
counts go to tests/golden/e2e_e2b_spec_ref.npz.

A third case runs the engine as a server (ENGINE_SERVE=1, one request per input line) through its
prefix cache with three conversation slots (ENGINE_SLOTS=3, ENGINE_SLOT_MIN_REUSE=32, :1569-1613):
continuation, switch, eviction and repeat (serve_requests).  Per request the tokens and TIMING's
reused= and slot= go to tests/golden/e2e_e2b_serve_ref.npz, against tests/oracle_lib.py's
OracleConversations, the restated policy the GPU request tests use.  A fourth case repeats the
speculative one after ENGINE_FAKE_CTX=600 positions of the engine's seeded K/V (fake), into
tests/golden/e2e_e2b_fake_ref.npz.

Needs ~16 GB of host memory (the serve case ~25 GB: one oracle model per slot) and ~7 GB of
temporary disk; run by hand (every case, or one of them):

    python tests/golden/make_golden_e2b.py [greedy|spec|serve|fake]
"""
import json
import os
import pathlib
import re
import struct
import subprocess
import sys
import tempfile
import time

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE.parent))

from oracle_lib import OracleConversations, OracleModel, e2e_config, make_prompt  # noqa: E402
from test_checkpoint import make_index  # noqa: E402

SEED = 20261202
N_PROMPT, N_NEW, N_REQ = 100, 8, 4
# the reference's hard-coded model (gemma4_engine.cpp:1222-1231, ENGINE_SPEC.md dimensions)
E2B = dict(hidden=1536, n_layers=35, mlp=6144, mlp_shared=12288, vocab=262144, kv_owners=15, ple=1, hd_global=512,
           rope_global_quarter=1, drafter=0, k_draft=0, ngram=0, prefill_int8=1, decode_int8=1, ctx_max=1024,
           prefill_block=32, seed=SEED)
SCALARS = {3: 0.75, 14: 1.5, 22: 0.5, 34: 1.25}  # a few layer scalars other than 1 (bf16 values)
# the speculative case: prompt lookup only (the oracle has no drafter here; the reference's is capped
# at 0 steps), verify passes past the split-KV threshold
SPEC = dict(ngram=2, ngram_len=3, k_draft=0)
SPEC_PROMPT, SPEC_NEW, SPEC_REQ = 220, 24, 3
# the fake-context case: ENGINE_FAKE_CTX positions of seeded K/V before the prompt
FAKE_N, FAKE_PROMPT, FAKE_NEW = 600, 60, 16
FAKE_SEEDS = (204, 205)  # prompts that do not lead to the random model's most frequent token
# the serve case: conversation slots (ENGINE_SLOTS) and their reuse threshold (ENGINE_SLOT_MIN_REUSE)
SERVE_SLOTS, SERVE_MIN_REUSE, SERVE_NEW = 3, 32, 4


def e2b_oracle(scalars=True, **over):
    m = OracleModel(e2e_config(**dict(E2B, **over)))
    if scalars:
        for l, v in SCALARS.items():
            m.set_layer_scalar(l, v)
    return m


def prompts():
    return [make_prompt(SEED % 1000 + i, N_PROMPT) for i in range(N_REQ)]


def spec_prompts():
    return [make_prompt(SEED % 1000 + 100 + i, SPEC_PROMPT) for i in range(SPEC_REQ)]


def fake_prompts():
    return [make_prompt(SEED % 1000 + s, FAKE_PROMPT) for s in FAKE_SEEDS]


def serve_requests():
    """A session through the prefix cache: a new conversation, its continuation, an unrelated one
    (a stored slot takes it), a return to the first sharing 50 tokens (switch), a prompt sharing
    fewer than SERVE_MIN_REUSE tokens with everything (the least recently used slot is evicted),
    and a repeat of the previous prompt (only its last token is re-run)."""
    a = make_prompt(SEED % 1000 + 204, 60)  # seeds whose prompts do not lead to the random model's
    b = make_prompt(SEED % 1000 + 207, 40)  # most frequent token (236283)
    extra = make_prompt(SEED % 1000 + 203, 60)
    return [a, np.concatenate([a, extra[:20]]), b, np.concatenate([a[:50], extra[20:30]]),
            np.concatenate([a[:10], extra[30:60]]), np.concatenate([a[:10], extra[30:60]])]


def write_placeholder_drafter(d):
    """A model.safetensors and index with the names the engine's drafter loader reads (:1519-1528):
    tiny bf16 tensors (2-D where it takes a shape) and the int64 token ordering."""
    d.mkdir(parents=True, exist_ok=True)
    tensors = {}
    for l in range(4):
        p = f"model.layers.{l}."
        for n in ("self_attn.q_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            tensors[p + n + ".weight"] = ("BF16", (1, 8))
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm", "self_attn.q_norm"):
            tensors[p + n + ".weight"] = ("BF16", (8,))
        tensors[p + "layer_scalar"] = ("BF16", (1,))
    for n in ("pre_projection.weight", "post_projection.weight", "masked_embedding.centroids.weight",
              "model.embed_tokens.weight"):
        tensors[n] = ("BF16", (1, 8))
    tensors["model.norm.weight"] = ("BF16", (8,))
    tensors["masked_embedding.token_ordering"] = ("I64", (16,))
    hdr, off = {}, 0
    for name, (dt, shape) in tensors.items():
        nb = int(np.prod(shape)) * (2 if dt == "BF16" else 8)
        hdr[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + nb]}
        off += nb
    h = json.dumps(hdr).encode()
    h += b" " * (-len(h) % 8)
    (d / "model.safetensors").write_bytes(struct.pack("<Q", len(h)) + h + bytes(off))
    make_index(d / "model.safetensors", d / "index.tsv")


def run_engine(binary, d, prompt, n_new, env):
    (d / "prompt.txt").write_text(" ".join(str(int(t)) for t in prompt))
    proc = subprocess.run([str(binary), str(d), str(d / "index.tsv"), str(d / "prompt.txt"), str(n_new)],
                          capture_output=True, text=True, env=env, timeout=3600)
    if proc.returncode != 0:
        sys.exit(proc.stderr[-3000:])
    gen = next(ln for ln in proc.stdout.splitlines() if ln.startswith("GEN:"))
    timing = next(ln for ln in proc.stdout.splitlines() if ln.startswith("TIMING"))
    ng = re.search(r"ngram_rounds=(\d+)/(\d+)", timing)
    return [int(x) for x in gen.split()[1:]], (int(ng.group(1)), int(ng.group(2)))


def greedy(binary, d, m, env):
    ps = prompts()
    gens = []
    for i, p in enumerate(ps):  # one run per prompt: each prefill starts at position 0
        t1 = time.time()
        gen, _ = run_engine(binary, d, p, N_NEW, dict(env, ENGINE_K="0"))
        print(f"reference engine, prompt {i}: {time.time() - t1:.0f} s", flush=True)
        gens.append(gen)
    ours = [[int(t) for t in m.generate(p, N_NEW)[0]] for p in ps]
    for g, o in zip(gens, ours):
        print("reference:", g, "\noracle:   ", o)
    for name, over in (("without per-layer embeddings", dict(ple=0)), ("every layer scalar 1", dict(scalars=False))):
        v = e2b_oracle(**over)
        firsts = [int(v.generate(p, 1)[0][0]) for p in ps]
        v.close()
        print(f"first tokens {name}: {firsts} (reference: {[g[0] for g in gens]})")
    # the float path end to end: ENGINE_PREFILL_INT8=0 and ENGINE_DECODE_INT8=0 (the reference's
    # fused float tasks for the MLP and the per-layer embeddings, :1267-1269, 1365-1366, 1380-1382)
    fgens = [run_engine(binary, d, p, N_NEW, dict(env, ENGINE_K="0", ENGINE_PREFILL_INT8="0",
                                                  ENGINE_DECODE_INT8="0"))[0] for p in ps]
    f = e2b_oracle(prefill_int8=0, decode_int8=0)
    fours = [[int(t) for t in f.generate(p, N_NEW)[0]] for p in ps]
    f.close()
    for g, o in zip(fgens, fours):
        print("reference (float):", g, "\noracle (float):   ", o)

    def pad(gs):
        tok = np.full((N_REQ, max(len(g) for g in gs)), -1, np.int32)
        for i, g in enumerate(gs):
            tok[i, :len(g)] = g
        return tok
    np.savez(HERE / "e2e_e2b_ref.npz", prompts=np.stack([np.asarray(p, np.int32) for p in ps]), tokens=pad(gens),
             tokens_float=pad(fgens), seed=SEED, n_new=N_NEW, scalar_layers=np.array(list(SCALARS), np.int32),
             scalar_values=np.array(list(SCALARS.values()), np.float32))
    print("greedy: agree" if ours == gens else "greedy: DIFFER")
    print("greedy float: agree" if fours == fgens else "greedy float: DIFFER")


def spec(binary, d, env):
    """Both decode modes: int8 verify passes (the default) and ENGINE_DECODE_INT8=0 (:1600, the float
    W4G32 path the reference's exactness claim is about); keys without and with the _dec0 suffix."""
    ps = spec_prompts()
    write_placeholder_drafter(d / "drafter")
    env = dict(env, ENGINE_K="3", ENGINE_POLICY="0,0,0", ENGINE_NGRAM=str(SPEC["ngram"]),
               ENGINE_NGLEN=str(SPEC["ngram_len"]), ENGINE_DRAFTER_DIR=str(d / "drafter"),
               ENGINE_DRAFTER_INDEX=str(d / "drafter" / "index.tsv"))
    out = dict(prompts=np.stack([np.asarray(p, np.int32) for p in ps]), seed=SEED, n_new=SPEC_NEW)
    for dec in (1, 0):
        sfx = "" if dec else "_dec0"
        gens, counts = [], []
        for i, p in enumerate(ps):
            t1 = time.time()
            gen, ng = run_engine(binary, d, p, SPEC_NEW, dict(env, ENGINE_DECODE_INT8=str(dec)))
            print(f"reference engine, speculative prompt {i}, decode int8 {dec}: {time.time() - t1:.0f} s, "
                  f"ngram_rounds/rounds {ng}", flush=True)
            gens.append(gen)
            counts.append(ng)
        m = e2b_oracle(decode_int8=dec, **SPEC)
        ours, ocounts = [], []
        for p in ps:
            t, st = m.generate(p, SPEC_NEW)
            ours.append([int(x) for x in t])
            ocounts.append((st["ngram_rounds"], st["rounds"]))
        m.close()
        for g, o, c, oc in zip(gens, ours, counts, ocounts):
            print("reference:", g, c, "\noracle:   ", o, oc)
        tok = np.full((SPEC_REQ, max(len(g) for g in gens)), -1, np.int32)
        for i, g in enumerate(gens):
            tok[i, :len(g)] = g
        out["tokens" + sfx] = tok
        out["ngram_rounds" + sfx] = np.array([c[0] for c in counts], np.int32)
        out["rounds" + sfx] = np.array([c[1] for c in counts], np.int32)
        print(f"speculative, decode int8 {dec}: " + ("agree" if (ours, ocounts) == (gens, counts) else "DIFFER"))
    np.savez(HERE / "e2e_e2b_spec_ref.npz", **out)


def serve(binary, d, env):
    """ENGINE_SERVE=1: one engine process, one request per stdin line ("<n_new> <tokens>", :1681-1689);
    per request the GEN tokens and TIMING's reused= and slot= fields."""
    reqs = serve_requests()
    env = dict(env, ENGINE_K="0", ENGINE_SERVE="1", ENGINE_SLOTS=str(SERVE_SLOTS),
               ENGINE_SLOT_MIN_REUSE=str(SERVE_MIN_REUSE))
    lines = "".join(f"{SERVE_NEW} " + " ".join(str(int(t)) for t in p) + "\n" for p in reqs)
    t1 = time.time()
    proc = subprocess.run([str(binary), str(d), str(d / "index.tsv"), "/dev/null", "0"], input=lines,
                          capture_output=True, text=True, env=env, timeout=3600)
    if proc.returncode != 0:
        sys.exit(proc.stderr[-3000:])
    gens = [[int(x) for x in ln.split()[1:]] for ln in proc.stdout.splitlines() if ln.startswith("GEN:")]
    timing = [ln for ln in proc.stdout.splitlines() if ln.startswith("TIMING")]
    reused = [int(re.search(r"reused=(\d+)", ln).group(1)) for ln in timing]
    slots = [int(re.search(r"slot=(\d+)", ln).group(1)) for ln in timing]
    print(f"reference engine, serve session: {time.time() - t1:.0f} s; reused {reused}, slots {slots}", flush=True)
    conv = OracleConversations(e2b_oracle, SERVE_SLOTS, SERVE_MIN_REUSE)
    ours = [conv.request(p, SERVE_NEW) for p in reqs]
    conv.close()
    for g, r, sl, o in zip(gens, reused, slots, ours):
        print("reference:", g, r, sl, "\noracle:   ", o[0], o[1], o[2])
    tok = np.full((len(reqs), SERVE_NEW), -1, np.int32)
    req = np.full((len(reqs), max(len(p) for p in reqs)), -1, np.int32)
    for i, (g, p) in enumerate(zip(gens, reqs)):
        tok[i, :len(g)] = g
        req[i, :len(p)] = p
    np.savez(HERE / "e2e_e2b_serve_ref.npz", requests=req, tokens=tok, reused=np.array(reused, np.int32),
             slot=np.array(slots, np.int32), seed=SEED, n_new=SERVE_NEW, slots=SERVE_SLOTS,
             min_reuse=SERVE_MIN_REUSE)
    same = [(o[0], o[1], o[2]) for o in ours] == list(zip(gens, reused, slots))
    print("serve: agree" if same else "serve: DIFFER")


def fake(binary, d, env):
    """ENGINE_FAKE_CTX=600 (:1249-1250): the owners' K/V rows of positions 0..599 filled from the
    engine's seeded LCG, the prompt at 600 on, speculative rounds with prompt lookup as above, so the
    verify passes attend ~680 keys through the split-KV attention."""
    ps = fake_prompts()
    write_placeholder_drafter(d / "drafter")
    env = dict(env, ENGINE_K="3", ENGINE_POLICY="0,0,0", ENGINE_NGRAM=str(SPEC["ngram"]),
               ENGINE_NGLEN=str(SPEC["ngram_len"]), ENGINE_DRAFTER_DIR=str(d / "drafter"),
               ENGINE_DRAFTER_INDEX=str(d / "drafter" / "index.tsv"), ENGINE_FAKE_CTX=str(FAKE_N))
    gens, counts = [], []
    for i, p in enumerate(ps):
        t1 = time.time()
        gen, ng = run_engine(binary, d, p, FAKE_NEW, env)
        print(f"reference engine, fake-context prompt {i}: {time.time() - t1:.0f} s, ngram_rounds/rounds {ng}",
              flush=True)
        gens.append(gen)
        counts.append(ng)
    m = e2b_oracle(**SPEC)
    m.fake_ctx(FAKE_N)
    ours, ocounts = [], []
    for p in ps:
        t, st = m.generate(p, FAKE_NEW)
        ours.append([int(x) for x in t])
        ocounts.append((st["ngram_rounds"], st["rounds"]))
    m.close()
    for g, o, c, oc in zip(gens, ours, counts, ocounts):
        print("reference:", g, c, "\noracle:   ", o, oc)
    tok = np.full((len(ps), FAKE_NEW), -1, np.int32)
    for i, g in enumerate(gens):
        tok[i, :len(g)] = g
    np.savez(HERE / "e2e_e2b_fake_ref.npz", prompts=np.stack([np.asarray(p, np.int32) for p in ps]), tokens=tok,
             seed=SEED, n_new=FAKE_NEW, fake_n=FAKE_N, ngram_rounds=np.array([c[0] for c in counts], np.int32),
             rounds=np.array([c[1] for c in counts], np.int32))
    print("fake context: agree" if (ours, ocounts) == (gens, counts) else "fake context: DIFFER")


def main():
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    binary = ROOT / "oracle" / "_ref" / "gemma4_engine"
    if not binary.exists():
        sys.exit(f"{binary} missing: make -C oracle engine REF=<reference checkout>")
    t0 = time.time()
    m = e2b_oracle()
    print(f"oracle model built in {time.time() - t0:.0f} s", flush=True)
    env = dict(os.environ, ENGINE_PREFILL_INT8="1", ENGINE_CTX="1024",
               ENGINE_CPUS=",".join(str(i) for i in range(min(8, os.cpu_count() or 1))))
    with tempfile.TemporaryDirectory() as d:
        d = pathlib.Path(d)
        m.write_checkpoint(d / "model.safetensors")
        make_index(d / "model.safetensors", d / "index.tsv")
        if which in ("all", "greedy"):
            greedy(binary, d, m, env)
        m.close()
        if which in ("all", "spec"):
            spec(binary, d, env)
        if which in ("all", "serve"):
            serve(binary, d, env)
        if which in ("all", "fake"):
            fake(binary, d, env)


if __name__ == "__main__":
    main()
