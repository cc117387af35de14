"""GGUF tensor ingestion (hayai_b200/gguf.py): files written by gguf-py's GGUFWriter (a
third-party writer pinned by this image) are read back tensor for tensor, malformed files are
rejected as the reference's parser rejects them (crates/hayai-model/src/gguf.rs:24-121), and on
the GPU an FFN stack loaded from a file matches the oracle on the same bytes."""
import struct

import numpy as np
import pytest
import torch

import oracle
from hayai_b200 import gguf as hg
from tests.helpers import assert_parity, quantized

EPS = 1e-5


def write_gguf(path, tensors, meta=None):
    """tensors: name -> (ggml type, ncols, nrows, bytes or f32 array)."""
    gguf = pytest.importorskip("gguf")
    w = gguf.GGUFWriter(str(path), "llama")
    for k, v in (meta or {}).items():
        w.add_uint32(k, v)
    for name, (t, ncols, nrows, data) in tensors.items():
        if t == oracle.F32:
            w.add_tensor(name, np.asarray(data, np.float32).reshape(nrows, ncols) if nrows > 1 else
                         np.asarray(data, np.float32))
        else:
            qk, bs = oracle.BLOCK[t]
            w.add_tensor(name, np.asarray(data, np.uint8).reshape(nrows, ncols // qk * bs),
                         raw_dtype=gguf.GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_reads_back_every_tensor(tmp_path):
    tens = {
        "blk.0.ffn_gate.weight": (oracle.Q4_K, 512, 96, quantized(oracle.Q4_K, 96, 512, 1)),
        "blk.0.ffn_down.weight": (oracle.Q6_K, 256, 64, quantized(oracle.Q6_K, 64, 256, 2)),
        "blk.0.attn_q.weight": (oracle.Q8_0, 64, 32, quantized(oracle.Q8_0, 32, 64, 3)),
        "blk.0.ffn_up.weight": (oracle.Q5_K, 512, 16, quantized(oracle.Q5_K, 16, 512, 4)),
        "blk.0.ffn_norm.weight": (oracle.F32, 256, 1, oracle.normal(5, 256)),
    }
    p = tmp_path / "m.gguf"
    write_gguf(p, tens, {"llama.block_count": 1})
    g = hg.GgufFile.open(p)
    try:
        assert g.version in (2, 3)
        assert g.metadata["general.architecture"] == "llama"
        assert g.metadata["llama.block_count"] == 1
        assert g.data_offset % g.alignment == 0
        for name, (t, ncols, nrows, data) in tens.items():
            info = g.tensor(name)
            assert (info.type_id, info.ncols, info.nrows) == (t, ncols, nrows)
            if t == oracle.F32:
                assert np.array_equal(g.f32(name), np.asarray(data, np.float32))
            else:
                assert np.array_equal(g.tensor_bytes(info), data)
                qm = g.load_quant_matrix(name)
                assert (qm.ncols, qm.nrows, qm.ggml_type) == (ncols, nrows, t)
                assert np.array_equal(qm.data, data)
        with pytest.raises(hg.GgufError):
            g.tensor("blk.9.ffn_gate.weight")
        with pytest.raises(hg.GgufError):
            g.f32("blk.0.ffn_gate.weight")
    finally:
        g.close()


def _header(version=3, n_tensors=1, n_kv=0, tensors=b"", kv=b"", magic=hg.GGUF_MAGIC):
    return struct.pack("<IIQQ", magic, version, n_tensors, n_kv) + kv + tensors


def _tensor_entry(name, dims, t=0, offset=0):
    b = name.encode()
    return struct.pack("<Q", len(b)) + b + struct.pack("<I", len(dims)) + b"".join(
        struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", t, offset)


@pytest.mark.parametrize("blob,what", [
    (_header(magic=0x12345678) + b"\0" * 64, "magic"),
    (_header(version=7) + b"\0" * 64, "version"),
    (_header(n_tensors=1 << 40) + b"\0" * 64, "count"),
    (_header(tensors=_tensor_entry("a", [4, 0, 1])) + b"\0" * 64, "zero dimension"),
    (_header(tensors=_tensor_entry("a", [1, 1, 1, 1, 1])) + b"\0" * 64, "dims"),
    (_header(n_tensors=2, tensors=_tensor_entry("a", [4]) + _tensor_entry("a", [4])) + b"\0" * 64, "duplicate"),
    (_header(n_kv=1, kv=struct.pack("<Q", 17) + b"general.alignment" + struct.pack("<II", 4, 24),
             tensors=_tensor_entry("a", [4])) + b"\0" * 64, "alignment"),
    (_header(tensors=_tensor_entry("a", [1 << 20])) + b"\0" * 64, "out of bounds"),
    # sizes and ranges are validated while the directory is parsed (gguf.rs:85-115)
    (_header(tensors=_tensor_entry("a", [4], t=99)) + b"\0" * 64, "unsupported ggml type"),
    (_header(tensors=_tensor_entry("a", [1 << 40, 1 << 40])) + b"\0" * 64, "element count overflow"),
    (_header(tensors=_tensor_entry("a", [(1 << 62) + 1], t=0)) + b"\0" * 64, "byte size overflow"),
    (_header(tensors=_tensor_entry("a", [4], offset=(1 << 64) - 1)) + b"\0" * 64, "absolute offset overflow"),
    (_header(tensors=_tensor_entry("a", [4], offset=(1 << 64) - 70)) + b"\0" * 64, "byte range overflow"),
    (_header()[:20], "truncated"),
])
def test_rejects_malformed_files(tmp_path, blob, what):
    p = tmp_path / "bad.gguf"
    p.write_bytes(blob)
    with pytest.raises(hg.GgufError) as e:
        g = hg.GgufFile.open(p)
        for t in g.tensors:  # a directory entry past the file end fails on access
            g.tensor_bytes(t)
    assert what in str(e.value)


@pytest.mark.gpu
def test_ffn_stack_from_gguf_file(tmp_path, engine):
    """Llama-3-8B-shaped FFN (reduced width) stored as a GGUF file, loaded and run as a stack."""
    L, dm, ff = 2, 1024, 2816
    tens, layers, norms = {}, [], []
    for l in range(L):
        g, u = quantized(oracle.Q4_K, ff, dm, 40 + l), quantized(oracle.Q4_K, ff, dm, 50 + l)
        d = quantized(oracle.Q6_K, dm, ff, 60 + l)
        nw = oracle.normal(70 + l, dm, 1.0, 0.1)
        tens[f"blk.{l}.ffn_gate.weight"] = (oracle.Q4_K, dm, ff, g)
        tens[f"blk.{l}.ffn_up.weight"] = (oracle.Q4_K, dm, ff, u)
        tens[f"blk.{l}.ffn_down.weight"] = (oracle.Q6_K, ff, dm, d)
        tens[f"blk.{l}.ffn_norm.weight"] = (oracle.F32, dm, 1, nw)
        layers.append((g, u, d))
        norms.append(nw)
    p = tmp_path / "ffn.gguf"
    write_gguf(p, tens)
    gf = hg.GgufFile.open(p)
    try:
        G, U, D, N = [], [], [], []
        for l in range(L):
            g, u, d, nw = gf.load_ffn_layer(engine, l)
            G.append(g)
            U.append(u)
            D.append(d)
            N.append(torch.from_numpy(nw).cuda())
    finally:
        gf.close()
    x = oracle.normal(80, dm)
    got = engine.ffn_stack(G, U, D, x, norms=N, eps=EPS)
    ref = x.copy()
    for (g, u, d), nw in zip(layers, norms):
        xn = oracle.rms_norm(ref, nw, EPS)
        ref = (ref + oracle.ffn_swiglu(oracle.Q4_K, g, oracle.Q4_K, u, oracle.Q6_K, d, dm, ff, dm, xn)).astype(np.float32)
    assert_parity(ref, got, what="stack loaded from GGUF")


def test_metadata_value_types(tmp_path):
    """Every metadata value type the reference reads (gguf.rs:633-672): scalars, bool, string,
    and (nested) arrays, as gguf-py writes them."""
    gguf = pytest.importorskip("gguf")
    p = tmp_path / "meta.gguf"
    w = gguf.GGUFWriter(str(p), "llama")
    w.add_uint32("t.u32", 7)
    w.add_int32("t.i32", -3)
    w.add_float32("t.f32", 0.25)
    w.add_uint64("t.u64", 1 << 40)
    w.add_bool("t.bool", True)
    w.add_string("t.str", "héllo")
    w.add_array("t.arr", [1, 2, 3])
    w.add_array("t.strs", ["a", "bc"])
    w.add_tensor("x", np.arange(8, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = hg.GgufFile.open(p)
    try:
        m = g.metadata
        assert (m["t.u32"], m["t.i32"], m["t.f32"], m["t.u64"], m["t.bool"]) == (7, -3, 0.25, 1 << 40, True)
        assert m["t.str"] == "héllo"
        assert m["t.arr"] == [1, 2, 3] and m["t.strs"] == ["a", "bc"]
        assert np.array_equal(g.f32("x"), np.arange(8, dtype=np.float32))
    finally:
        g.close()


def test_parser_rejects_arbitrary_bytes_cleanly(tmp_path):
    """Truncations and byte flips of a valid file: the parser either succeeds or raises
    GgufError, never another exception (the reference's hostile-input guards, gguf.rs:39-48)."""
    hyp = pytest.importorskip("hypothesis")
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    src = tmp_path / "ok.gguf"
    write_gguf(src, {"blk.0.ffn_gate.weight": (oracle.Q4_K, 256, 16, quantized(oracle.Q4_K, 16, 256, 9)),
                     "blk.0.ffn_norm.weight": (oracle.F32, 256, 1, oracle.normal(10, 256))}, {"llama.block_count": 1})
    good = src.read_bytes()
    bad = tmp_path / "fuzz.gguf"

    @settings(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
    @given(cut=st.integers(0, len(good)), flips=st.lists(st.tuples(st.integers(0, len(good) - 1),
                                                                   st.integers(0, 255)), max_size=6))
    def check(cut, flips):
        b = bytearray(good[:max(cut, 0)])
        for pos, val in flips:
            if pos < len(b):
                b[pos] = val
        bad.write_bytes(bytes(b))
        try:
            g = hg.GgufFile.open(bad)
        except hg.GgufError:
            return
        try:
            for t in g.tensors:
                try:
                    g.tensor_bytes(t)
                except hg.GgufError:
                    pass
        finally:
            g.close()

    assert hyp is not None
    check()
