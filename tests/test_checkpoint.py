"""The checkpoint reader (g4_checkpoint_* in include/g4.h) on the host, no GPU: checkpoints in the
reference's format written from the oracle's synthetic model, read through the safetensors header
and through the reference's index file (tools/make_index.py's lines, restated below and, where the
reference tree is present, checked against that tool's own output), the model sizes they give, and
the errors for damaged files and for parts of the real E2B model this build does not run."""
import json
import os
import pathlib
import struct
import subprocess
import sys

import numpy as np
import pytest

from g4pkg import g4
from oracle_lib import OracleModel, e2e_config

SMALL = dict(hidden=512, n_layers=5, mlp=1024, vocab=4096, ctx_max=1024)
# the reference checkout: G4_REFERENCE, else a "reference" directory beside this repository
REFERENCE_TOOL = pathlib.Path(os.environ.get("G4_REFERENCE", str(pathlib.Path(__file__).resolve().parents[2] /
                                                                  "reference"))) / "tools" / "make_index.py"


def make_index(src, out):
    """tools/make_index.py:1-9: one line per tensor of the safetensors header - name, dtype, absolute
    offset (8 + header length + the tensor's first data offset), byte count, comma-joined shape."""
    with open(src, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        hdr = json.loads(fh.read(n))
    with open(out, "w") as o:
        for k, v in hdr.items():
            if k == "__metadata__":
                continue
            a, b = v["data_offsets"]
            o.write(f"{k}\t{v['dtype']}\t{8 + n + a}\t{b - a}\t{','.join(map(str, v['shape']))}\n")


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    m = OracleModel(e2e_config(**SMALL, seed=777))
    try:
        m.set_layer_scalar(1, 0.5)
        m.set_layer_scalar(3, 1.25)
        m.write_checkpoint(d / "model.safetensors")
        m.write_checkpoint(d / "u8.safetensors", packed_u8=True)
    finally:
        m.close()
    make_index(d / "model.safetensors", d / "index.tsv")
    return d


def read_index(path):
    return [line.rstrip("\n").split("\t") for line in open(path) if line.strip()]


def write_index(path, rows):
    with open(path, "w") as f:
        for r in rows:
            f.write("\t".join(r) + "\n")


def test_header_and_index_agree(ckpt):
    a = g4.Checkpoint(ckpt)  # the directory, as the reference's <ckpt> argument
    b = g4.Checkpoint(ckpt / "model.safetensors", ckpt / "index.tsv")
    try:
        rows = read_index(ckpt / "index.tsv")
        assert len(a) == len(b) == len(rows) == 5 * (14 + 7) + 2
        for name, dtype, off, nb, shape in rows:
            want = (dtype, tuple(int(x) for x in shape.split(",") if x), int(nb))
            assert a.tensor(name) == want == b.tensor(name), name
        assert a.tensor("layers.0.self_attn.q_proj.weight_packed") == ("I32", (2048, 64), 2048 * 256)
        assert a.tensor("layers.2.mlp.down_proj.weight_scale") == ("BF16", (512, 32), 512 * 32 * 2)
        assert a.tensor("embed_tokens.weight") == ("BF16", (4096, 512), 4096 * 512 * 2)
    finally:
        a.close()
        b.close()


@pytest.mark.skipif(not REFERENCE_TOOL.exists(), reason="the reference tree is not on this machine")
def test_index_restatement_matches_the_reference_tool(ckpt, tmp_path):
    out = tmp_path / "ref_index.tsv"
    subprocess.run([sys.executable, str(REFERENCE_TOOL), str(ckpt / "model.safetensors"), str(out)], check=True,
                   capture_output=True)
    assert out.read_text() == (ckpt / "index.tsv").read_text()


@pytest.mark.parametrize("name", ["model.safetensors", "u8.safetensors"])
def test_config_gives_the_model_sizes(ckpt, name):
    ck = g4.Checkpoint(ckpt / name)
    try:
        cfg = ck.config(hidden=2048, n_layers=30, mlp=8192, vocab=262144)
        assert (cfg.hidden, cfg.n_layers, cfg.mlp, cfg.vocab) == (512, 5, 1024, 4096)
        assert cfg.ctx_max == g4.engine_config().ctx_max  # other fields untouched
    finally:
        ck.close()


def test_layer_scalars_are_stored_as_bf16(ckpt):
    data = (ckpt / "model.safetensors").read_bytes()
    n = struct.unpack("<Q", data[:8])[0]
    hdr = json.loads(data[8:8 + n])
    vals = []
    for l in range(5):
        a, b = hdr[f"layers.{l}.layer_scalar"]["data_offsets"]
        bits = np.frombuffer(data[8 + n + a:8 + n + b], np.uint16)
        vals.append(float((bits.astype(np.uint32) << 16).view(np.float32)[0]))
    assert vals == [1.0, 0.5, 1.0, 1.25, 1.0]


def expect_error(fn, code, words):
    with pytest.raises(RuntimeError) as ei:
        fn()
    msg = str(ei.value)
    for w in words:
        assert w in msg, msg
    return msg


def test_missing_tensor_is_named(ckpt, tmp_path):
    rows = [r for r in read_index(ckpt / "index.tsv") if r[0] != "layers.2.mlp.up_proj.weight_scale"]
    write_index(tmp_path / "i.tsv", rows)
    ck = g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "i.tsv")
    try:
        expect_error(lambda: ck.config(), None, ["layers.2.mlp.up_proj.weight_scale", "missing"])
    finally:
        ck.close()


def test_wrong_shape_is_reported(ckpt, tmp_path):
    rows = read_index(ckpt / "index.tsv")
    for r in rows:
        if r[0] == "layers.1.self_attn.o_proj.weight_scale":  # same bytes, another shape
            r[4] = "256,128"
    write_index(tmp_path / "i.tsv", rows)
    ck = g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "i.tsv")
    try:
        expect_error(lambda: ck.config(), None, ["layers.1.self_attn.o_proj.weight_scale", "expected BF16 [512,64]"])
    finally:
        ck.close()


def test_damaged_files_fail_at_open(ckpt, tmp_path):
    rows = read_index(ckpt / "index.tsv")
    size = (ckpt / "model.safetensors").stat().st_size
    bad = [list(r) for r in rows]
    bad[3][2] = str(size - 8)  # past the end of the file
    write_index(tmp_path / "end.tsv", bad)
    expect_error(lambda: g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "end.tsv"), None, ["past the end"])
    bad = [list(r) for r in rows]
    bad[5][3] = str(int(bad[5][3]) - 2)  # byte count not dtype x shape
    write_index(tmp_path / "nb.tsv", bad)
    expect_error(lambda: g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "nb.tsv"), None, ["bytes"])
    trunc = tmp_path / "trunc.safetensors"
    trunc.write_bytes((ckpt / "model.safetensors").read_bytes()[:4096])
    expect_error(lambda: g4.Checkpoint(trunc), None, ["trunc.safetensors"])
    expect_error(lambda: g4.Checkpoint(tmp_path / "none.safetensors"), None, ["cannot open"])
    deep = ('{"__metadata__":' + "[" * 200 + "]" * 200 + "}").encode()  # nesting past the parser's bound
    deep += b" " * (-len(deep) % 8)
    (tmp_path / "deep.safetensors").write_bytes(struct.pack("<Q", len(deep)) + deep)
    expect_error(lambda: g4.Checkpoint(tmp_path / "deep.safetensors"), None, ["malformed"])


def test_e2b_parts_are_reported_unsupported(ckpt, tmp_path):
    rows = read_index(ckpt / "index.tsv")
    emb = next(r for r in rows if r[0] == "embed_tokens.weight")
    # a per-layer embedding table of the wrong width (here aliasing the embedding's bytes)
    write_index(tmp_path / "ple.tsv", rows + [["embed_tokens_per_layer.weight", "BF16", emb[2], emb[3], emb[4]]])
    ck = g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "ple.tsv")
    try:
        expect_error(lambda: ck.config(), None, ["embed_tokens_per_layer.weight", "expected BF16 [4096,1280]"])
    finally:
        ck.close()
    # a KV-shared layer without an owner of its type: layer 4 is the first global layer
    shared = [r for r in rows if not r[0].startswith(("layers.4.self_attn.k_proj", "layers.4.self_attn.v_proj"))]
    write_index(tmp_path / "kv.tsv", shared)
    ck = g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "kv.tsv")
    try:
        expect_error(lambda: ck.config(), None, ["KV-shared layer 4", "no global layer"])
    finally:
        ck.close()
    # k/v projections after a KV-shared layer
    gap = [r for r in rows if not r[0].startswith(("layers.2.self_attn.k_proj", "layers.2.self_attn.v_proj"))]
    write_index(tmp_path / "gap.tsv", gap)
    ck = g4.Checkpoint(ckpt / "model.safetensors", tmp_path / "gap.tsv")
    try:
        expect_error(lambda: ck.config(), None, ["layer 3 has k/v projections after the KV-shared layer 2"])
    finally:
        ck.close()


def test_ple_checkpoint(tmp_path):
    """Per-layer embeddings (the E2B model's PLE): the table [vocab][n_layers x 256], the projection of
    the embedding and its norm, and per layer the input gate, the projection and its norm; the
    config sets ple."""
    m = OracleModel(e2e_config(**SMALL, seed=779, ple=1))
    try:
        m.write_checkpoint(tmp_path / "model.safetensors")
    finally:
        m.close()
    ck = g4.Checkpoint(tmp_path)
    try:
        cfg = ck.config()
        assert (cfg.n_layers, cfg.ple, cfg.kv_owners) == (5, 1, 0)
        assert ck.tensor("embed_tokens_per_layer.weight")[:2] == ("BF16", (4096, 1280))
        assert ck.tensor("per_layer_model_projection.weight_packed")[:2] == ("I32", (1280, 64))
        assert ck.tensor("layers.3.per_layer_projection.weight_packed")[:2] == ("I32", (512, 32))
        assert ck.tensor("layers.3.post_per_layer_input_norm.weight")[:2] == ("BF16", (512,))
        # an engine from it is refused before any device work (the path is not verified)
        with pytest.raises(RuntimeError, match="per-layer embeddings from a checkpoint"):
            g4.Engine(g4.engine_config(), checkpoint=ck)
    finally:
        ck.close()


def _bf16_tensor(path, name):
    data = pathlib.Path(path).read_bytes()
    n = struct.unpack("<Q", data[:8])[0]
    a, b = json.loads(data[8:8 + n])[name]["data_offsets"]
    return np.frombuffer(data[8 + n + a:8 + n + b], np.uint16)


def test_ple_checkpoint_keeps_the_final_norm(tmp_path):
    """The per-layer projection norm is written after norm.weight, not over it: norm.weight is the
    same with and without per-layer embeddings (the final norm is generated independently of them)."""
    for ple in (0, 1):
        m = OracleModel(e2e_config(**SMALL, seed=780, ple=ple))
        try:
            m.write_checkpoint(tmp_path / f"ple{ple}.safetensors")
        finally:
            m.close()
    a = _bf16_tensor(tmp_path / "ple0.safetensors", "norm.weight")
    b = _bf16_tensor(tmp_path / "ple1.safetensors", "norm.weight")
    c = _bf16_tensor(tmp_path / "ple1.safetensors", "per_layer_projection_norm.weight")
    assert a.size == 512 and np.array_equal(a, b)
    assert not np.array_equal(b[:256], c)


def test_kv_shared_checkpoint(tmp_path):
    """Trailing layers without k/v projections (the E2B model's KV sharing, :1251): the config names
    the first of them as kv_owners and their (here doubled) MLP width as mlp_shared, and the shared
    layers carry no k_proj, v_proj or k_norm."""
    m = OracleModel(e2e_config(**dict(SMALL, n_layers=10), seed=778, kv_owners=5, mlp_shared=2048))
    try:
        m.write_checkpoint(tmp_path / "model.safetensors")
    finally:
        m.close()
    ck = g4.Checkpoint(tmp_path)
    try:
        cfg = ck.config()
        assert (cfg.n_layers, cfg.kv_owners, cfg.mlp, cfg.mlp_shared) == (10, 5, 1024, 2048)
        assert ck.tensor("layers.6.mlp.down_proj.weight_scale")[1] == (512, 64)
        assert len(ck) == 5 * 21 + 5 * 16 + 2
        expect_error(lambda: ck.tensor("layers.7.self_attn.k_proj.weight_packed"), None, ["no tensor"])
        assert ck.tensor("layers.7.self_attn.q_proj.weight_packed")[1] == (2048, 64)
    finally:
        ck.close()
