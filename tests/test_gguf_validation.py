"""The engine's GGUF reader and model check on malformed files (no GPU).

`lfm_model_inspect` runs the checks of `lfm_engine_create` that need no
device: the header rules of the reference parser (parser/src/gguf.rs:304-440,
its tests from :573), the hyperparameter check of load_hyperparams
(engine/src/lfm.rs:102-145, typed metadata of engine/src/model_file.rs:131-182)
and the tensor table the engine loads. Each case builds a small file on the
host and expects LFM_ERR_MODEL with the reference's message. The positive case
is the synthetic model's full header over a sparse file of the model's size.
"""

import ctypes
import os
import struct

import pytest

import synth_gguf as sg

LFM_ERR_MODEL = 2


def kv_u32(k, v):
    b = k.encode()
    return struct.pack("<Q", len(b)) + b + struct.pack("<II", sg.T_U32, v)


def kv_raw(k, vtype, payload):
    b = k.encode()
    return struct.pack("<Q", len(b)) + b + struct.pack("<I", vtype) + payload


def tinfo(name, ne, gtype, offset):
    b = name.encode()
    return (struct.pack("<Q", len(b)) + b + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
            + struct.pack("<IQ", gtype, offset))


def gguf(kvs=(), tensors=(), version=3, magic=b"GGUF", n_tensors=None, n_kv=None, align=32, data=0):
    head = magic + struct.pack("<IQQ", version, len(tensors) if n_tensors is None else n_tensors,
                               len(kvs) if n_kv is None else n_kv)
    head += b"".join(kvs) + b"".join(tensors)
    pad = (-len(head)) % align
    return head + b"\0" * pad + b"\0" * data


def inspect(tmp_path, blob):
    import lfm2_b200
    p = tmp_path / "m.gguf"
    p.write_bytes(blob)
    hp = lfm2_b200.Hparams()
    st = lfm2_b200.lib().lfm_model_inspect(str(p).encode(), ctypes.byref(hp))
    return st, lfm2_b200.lib().lfm_global_error().decode(), hp


def expect(tmp_path, blob, msg):
    st, err, _ = inspect(tmp_path, blob)
    assert st == LFM_ERR_MODEL, (st, err)
    assert msg in err, err


# ---- header rules (parser/src/gguf.rs:304-440 and its tests)

def test_invalid_magic(tmp_path):
    expect(tmp_path, gguf(magic=b"GGUX"), "Invalid magic")


def test_invalid_version(tmp_path):
    expect(tmp_path, gguf(version=2), "Unsupported GGUF version: 2 (expected 3)")


def test_truncated_header(tmp_path):
    expect(tmp_path, b"GGUF" + struct.pack("<I", 3) + b"\1\0", "Unexpected end of file")


def test_counts_bounded(tmp_path):
    expect(tmp_path, gguf(n_tensors=100001), "Tensor count 100001 exceeds maximum")
    expect(tmp_path, gguf(n_kv=100001), "KV count 100001 exceeds maximum")


def test_duplicate_metadata_key(tmp_path):
    expect(tmp_path, gguf([kv_u32("a", 1), kv_u32("a", 2)]), "Duplicate metadata key: a")


def test_unknown_metadata_value_type(tmp_path):
    expect(tmp_path, gguf([kv_raw("k", 99, b"")]), "Unknown metadata value type: 99")


def test_invalid_bool(tmp_path):
    expect(tmp_path, gguf([kv_raw("k", sg.T_BOOL, b"\2")]), "Invalid BOOL value: 2")


def test_array_length_bounded(tmp_path):
    expect(tmp_path, gguf([kv_raw("k", sg.T_ARR, struct.pack("<IQ", sg.T_U8, 10_000_001))]),
           "Array length 10000001 exceeds maximum")


def test_string_length_bounded(tmp_path):
    expect(tmp_path, gguf([kv_raw("k", sg.T_STR, struct.pack("<Q", (1 << 30) + 1))]),
           "String length 1073741825 exceeds maximum (1 GiB)")


def test_invalid_utf8(tmp_path):
    bad = b"\xc0\xaf"  # overlong '/'
    expect(tmp_path, gguf([kv_raw("k", sg.T_STR, struct.pack("<Q", 2) + bad)]), "Invalid UTF-8")
    expect(tmp_path, gguf([kv_raw("k", sg.T_STR, struct.pack("<Q", 3) + b"\xed\xa0\x80")]), "Invalid UTF-8")


def test_alignment_power_of_two(tmp_path):
    expect(tmp_path, gguf([kv_u32("general.alignment", 48)]), "Invalid alignment: 48 (must be a power of two)")


def test_too_many_dimensions(tmp_path):
    expect(tmp_path, gguf(tensors=[tinfo("t", [1] * 9, 0, 0)]), "Too many dimensions: 9 (max 8)")


def test_unknown_ggml_type(tmp_path):
    expect(tmp_path, gguf(tensors=[tinfo("t", [10], 999, 0)], data=64), "Unknown GGML type: 999")


def test_q6k_block_multiple(tmp_path):
    expect(tmp_path, gguf(tensors=[tinfo("t", [100], 14, 0)], data=256),
           "Tensor has 100 elements, not a multiple of block size 256 for GGML type 14")


def test_overflowing_dimensions(tmp_path):
    expect(tmp_path, gguf(tensors=[tinfo("t", [2**64 - 1, 2], 0, 0)]), "overflow")


def test_duplicate_tensor_name(tmp_path):
    expect(tmp_path, gguf(tensors=[tinfo("t", [4], 0, 0), tinfo("t", [4], 0, 32)], data=64),
           "Duplicate tensor name: t")


def test_tensor_outside_file(tmp_path):
    # parser test_parse_out_of_file_storage: 1M f32 with no payload bytes
    expect(tmp_path, gguf(tensors=[tinfo("big", [1000000], 0, 0)]), 'Tensor "big" end 4000000 exceeds data size 0')
    expect(tmp_path, gguf(tensors=[tinfo("t", [4], 0, 4096)], data=32), 'Tensor "t" offset 4096 exceeds data size 32')


def test_empty_tensor_accepted_by_the_reader(tmp_path):
    # a zero-sized tensor parses (gguf.rs test_parse_empty_tensor); the model
    # check then fails on the hyperparameters, not on the header
    st, err, _ = inspect(tmp_path, gguf(tensors=[tinfo("empty", [0, 2048], 0, 0)]))
    assert st == LFM_ERR_MODEL and "metadata lfm2moe.block_count not a u32" in err, err


# ---- hyperparameters and the tensor table (lfm.rs:102-145)

def _model_header(tmp_path, meta_edit=None, plan_edit=None, sparse=True):
    """The synthetic model's header (its full metadata and tensor table) over
    a sparse file of the model's size: no payload is written."""
    kvs = sg.metadata(1234, sg.ATTN_LAYERS)
    if meta_edit:
        kvs = meta_edit(kvs)
    plan = sg.tensor_plan()
    if plan_edit:
        plan = plan_edit(plan)
    infos, off = [], 0
    for name, gtype, ne, _ in plan:
        infos.append(tinfo(name, list(ne), gtype, off))
        off += sg.nbytes_of(gtype, ne)
        off = (off + 31) // 32 * 32
    blob = gguf(kvs, infos)
    p = tmp_path / "model.gguf"
    p.write_bytes(blob)
    if sparse:
        os.truncate(p, len(blob) + off)
    return str(p)


def _inspect_path(path):
    import lfm2_b200
    hp = lfm2_b200.Hparams()
    st = lfm2_b200.lib().lfm_model_inspect(path.encode(), ctypes.byref(hp))
    return st, lfm2_b200.lib().lfm_global_error().decode(), hp


def _replace_u32(key, value):
    def edit(kvs):
        out = [kv for kv in kvs if not kv.startswith(struct.pack("<Q", len(key)) + key.encode() + struct.pack("<I", sg.T_U32))]
        assert len(out) == len(kvs) - 1, key
        return out + [kv_u32(key, value)]
    return edit


def test_full_header_passes(tmp_path):
    st, err, hp = _inspect_path(_model_header(tmp_path))
    assert st == 0, err
    assert (hp.dim, hp.heads, hp.n_layers, hp.vocab, hp.n_expert, hp.n_used, hp.expert_ff) == \
        (2048, 32, 24, 128000, 32, 4, 1792)
    assert [hp.kv_heads[l] for l in range(24)] == [8 if l in sg.ATTN_LAYERS else 0 for l in range(24)]
    assert hp.eos == sg.EOS_ID and abs(hp.eps - 1e-5) < 1e-12 and hp.rope_theta == 1e6


@pytest.mark.parametrize("key,value,field", [
    ("lfm2moe.vocab_size", 65536, "vocab=65536"),
    ("lfm2moe.expert_count", 16, "n_expert=16"),
    ("lfm2moe.expert_used_count", 8, "n_used=8"),
    ("lfm2moe.block_count", 16, "layers=16"),
    ("lfm2moe.embedding_length", 4096, "dim=4096"),
    ("lfm2moe.expert_feed_forward_length", 2048, "expert_ff=2048"),
])
def test_geometry_rejected(tmp_path, key, value, field):
    st, err, _ = _inspect_path(_model_header(tmp_path, meta_edit=_replace_u32(key, value)))
    assert st == LFM_ERR_MODEL and "unsupported geometry:" in err and field in err, err


def test_missing_metadata_key(tmp_path):
    key = "lfm2moe.attention.head_count"

    def drop(kvs):
        return [kv for kv in kvs if not kv.startswith(struct.pack("<Q", len(key)) + key.encode() + struct.pack("<I", sg.T_U32))]
    st, err, _ = _inspect_path(_model_header(tmp_path, meta_edit=drop))
    assert st == LFM_ERR_MODEL and "metadata lfm2moe.attention.head_count not a u32" in err, err


def test_missing_and_misshapen_tensors(tmp_path):
    st, err, _ = _inspect_path(_model_header(
        tmp_path, plan_edit=lambda pl: [t for t in pl if t[0] != "blk.5.ffn_down_exps.weight"]))
    assert st == LFM_ERR_MODEL and "missing tensor blk.5.ffn_down_exps.weight" in err, err
    st, err, _ = _inspect_path(_model_header(
        tmp_path, plan_edit=lambda pl: [(n, g, (2048, 256) if n == "blk.2.attn_k.weight" else ne, k)
                                        for n, g, ne, k in pl]))
    assert st == LFM_ERR_MODEL and "tensor blk.2.attn_k.weight has unexpected type/shape" in err, err


def test_truncated_model_file(tmp_path):
    """The header is whole but the payload is cut short: the last tensor ends
    past the end of the file (gguf.rs bounds check)."""
    p = _model_header(tmp_path)
    os.truncate(p, os.path.getsize(p) - 1)
    st, err, _ = _inspect_path(p)
    assert st == LFM_ERR_MODEL and 'Tensor "blk.23.ffn_down_exps.weight" end' in err, err


@pytest.mark.gpu
def test_engine_create_rejects_malformed_models(tmp_path, cuda_lib):
    """lfm_engine_create runs the same checks before it touches the device's
    memory: LFM_ERR_MODEL, no engine, the reference's message."""
    import lfm2_b200
    lib = lfm2_b200.lib()
    bad = tmp_path / "v2.gguf"
    bad.write_bytes(gguf(version=2))
    cases = [(str(bad), "Unsupported GGUF version: 2"),
             (_model_header(tmp_path, meta_edit=_replace_u32("lfm2moe.vocab_size", 65536)),
              "unsupported geometry: dim=2048 heads=32 layers=24 vocab=65536")]
    for path, msg in cases:
        h = ctypes.c_void_p()
        st = lib.lfm_engine_create(path.encode(), 0, ctypes.byref(h))
        assert st == LFM_ERR_MODEL and not h.value
        assert msg in lib.lfm_global_error().decode()
