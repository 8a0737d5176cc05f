"""GGUF reader (include/cfi_gguf.h) on files written by the package's writer: every metadata value
type, tensor types and dims, alignment, and the malformed files the reader must refuse.  Host-only
(no CUDA call)."""
import struct

import numpy as np
import pytest

import gguf as G

RNG = np.random.default_rng(7)


def sample_tensors():
    f32 = RNG.normal(size=(3, 8)).astype(np.float32)
    f16 = RNG.normal(size=16).astype(np.float16)
    q80 = RNG.integers(0, 256, size=5 * 2 * 34, dtype=np.uint8)          # 5 rows x 64 values
    q4k = RNG.integers(0, 256, size=2 * 144, dtype=np.uint8)             # 2 rows x 256 values
    return [("w.f32", 0, (8, 3), f32.tobytes()), ("w.f16", 1, (16,), f16.tobytes()),
            ("blk.0.attn_q.weight", 8, (64, 5), q80.tobytes()), ("blk.0.ffn_down.weight", 12, (256, 2), q4k.tobytes())]


KV = {
    "general.architecture": (G.STRING, "qwen2"),
    "u8": (G.U8, 200), "i8": (G.I8, -5), "u16": (G.U16, 60000), "i16": (G.I16, -300), "u32": (G.U32, 4000000000),
    "i32": (G.I32, -7), "f32": (G.F32, 1.5), "bool": (G.BOOL, True), "u64": (G.U64, 2 ** 40), "i64": (G.I64, -(2 ** 40)),
    "f64": (G.F64, 0.125), "arr.i32": (G.ARRAY, (G.I32, [1, -2, 3])),
    "tokenizer.ggml.tokens": (G.ARRAY, (G.STRING, ["a", "bc", "", "δ"])),
}


@pytest.mark.parametrize("alignment", [32, 64])
def test_round_trip(tmp_path, alignment):
    p = tmp_path / "m.gguf"
    ts = sample_tensors()
    G.write_gguf(p, KV, ts, alignment=alignment)
    with G.GGUFFile(p) as f:
        assert f.version == 3 and f.alignment == alignment
        for k, (t, v) in KV.items():
            got = f.get(k)
            want = list(v[1]) if t == G.ARRAY else v
            assert got == want, k
        assert f.get("missing", 42) == 42
        assert f.tensor_names() == [t[0] for t in ts]
        for name, ty, dims, data in ts:
            gty, gdims, arr = f.tensor(name)
            assert (gty, gdims) == (ty, dims)
            assert arr.tobytes() == data
        for i in range(len(ts)):
            assert f.info(i)[4] % alignment == 0  # data pointers aligned (the mapping is page aligned)


def _write(tmp_path, **kw):
    p = tmp_path / "m.gguf"
    G.write_gguf(p, {"general.architecture": (G.STRING, "x")}, sample_tensors(), **kw)
    return p, bytearray(p.read_bytes())


def test_refuses_bad_magic_version_and_truncation(tmp_path):
    p, b = _write(tmp_path)
    bad = bytearray(b)
    bad[0:4] = b"GGUX"
    (tmp_path / "a.gguf").write_bytes(bad)
    with pytest.raises(G.GGUFError, match="magic"):
        G.GGUFFile(tmp_path / "a.gguf")
    bad = bytearray(b)
    bad[4:8] = struct.pack("<I", 1)
    (tmp_path / "b.gguf").write_bytes(bad)
    with pytest.raises(G.GGUFError, match="version"):
        G.GGUFFile(tmp_path / "b.gguf")
    (tmp_path / "c.gguf").write_bytes(b[: len(b) - 200])
    with pytest.raises(G.GGUFError, match="past the end"):
        G.GGUFFile(tmp_path / "c.gguf")
    (tmp_path / "d.gguf").write_bytes(b[:40])
    with pytest.raises(G.GGUFError):
        G.GGUFFile(tmp_path / "d.gguf")
    with pytest.raises(G.GGUFError, match="cannot open"):
        G.GGUFFile(tmp_path / "nope.gguf")


def test_refuses_partial_blocks_and_misaligned_offsets(tmp_path):
    p, b = _write(tmp_path)
    name = b"blk.0.attn_q.weight"
    i = bytes(b).index(name) + len(name)  # then u32 n_dims, u64 ne0
    bad = bytearray(b)
    bad[i + 4:i + 12] = struct.pack("<Q", 48)  # 48 values: not whole Q8_0 blocks
    (tmp_path / "e.gguf").write_bytes(bad)
    with pytest.raises(G.GGUFError, match="whole blocks"):
        G.GGUFFile(tmp_path / "e.gguf")
    bad = bytearray(b)
    j = i + 4 + 8 * 2 + 4  # n_dims 2: past ne0, ne1 and the type: the offset
    off = struct.unpack("<Q", bytes(bad[j:j + 8]))[0]
    bad[j:j + 8] = struct.pack("<Q", off + 4)
    (tmp_path / "f.gguf").write_bytes(bad)
    with pytest.raises(G.GGUFError, match="aligned"):
        G.GGUFFile(tmp_path / "f.gguf")


def test_type_bytes():
    L = G._lib()
    assert L.cfi_gguf_type_bytes(8, 64) == 68
    assert L.cfi_gguf_type_bytes(12, 512) == 288
    assert L.cfi_gguf_type_bytes(14, 256) == 210
    assert L.cfi_gguf_type_bytes(8, 48) == 0
    assert L.cfi_gguf_type_bytes(99, 32) == 0
