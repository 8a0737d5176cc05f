"""GGUF model files: the reader of include/cfi_gguf.h (ctypes) and a small writer.

The reader maps the file through the library and hands out tensors as numpy views of ggml's block
bytes (no copy), ready for the device.  The writer emits GGUF v3 (metadata of scalars, strings and
arrays; tensors aligned to 32 bytes) -- enough to export a model of the decode driver or to build
test files; it follows the published GGUF layout that the reader checks.
"""
import ctypes as C
import struct

import numpy as np

import cfi_b200 as cfi

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}


def _lib():
    L = cfi.lib()
    if not getattr(L, "_gguf_ready", False):
        vp, i64, u64 = C.c_void_p, C.c_int64, C.c_uint64
        L.cfi_gguf_open.argtypes = [C.c_char_p, C.POINTER(vp), C.c_char_p, C.c_size_t]
        L.cfi_gguf_close.argtypes = [vp]
        L.cfi_gguf_close.restype = None
        L.cfi_gguf_version.argtypes = [vp]
        L.cfi_gguf_version.restype = C.c_uint32
        L.cfi_gguf_alignment.argtypes = [vp]
        L.cfi_gguf_alignment.restype = u64
        L.cfi_gguf_data_offset.argtypes = [vp]
        L.cfi_gguf_data_offset.restype = u64
        L.cfi_gguf_kv_count.argtypes = [vp]
        L.cfi_gguf_kv_count.restype = i64
        L.cfi_gguf_find_key.argtypes = [vp, C.c_char_p]
        L.cfi_gguf_find_key.restype = i64
        L.cfi_gguf_key.argtypes = [vp, i64]
        L.cfi_gguf_key.restype = C.c_char_p
        L.cfi_gguf_kv_type.argtypes = [vp, i64, C.POINTER(C.c_int), C.POINTER(u64)]
        L.cfi_gguf_get_i64.argtypes = [vp, i64, u64, C.POINTER(i64)]
        L.cfi_gguf_get_f64.argtypes = [vp, i64, u64, C.POINTER(C.c_double)]
        L.cfi_gguf_get_str.argtypes = [vp, i64, u64, C.POINTER(C.c_char_p), C.POINTER(u64)]
        L.cfi_gguf_tensor_count.argtypes = [vp]
        L.cfi_gguf_tensor_count.restype = i64
        L.cfi_gguf_find_tensor.argtypes = [vp, C.c_char_p]
        L.cfi_gguf_find_tensor.restype = i64
        L.cfi_gguf_tensor_info.argtypes = [vp, i64, C.POINTER(C.c_char_p), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                           C.POINTER(u64), C.POINTER(u64), C.POINTER(vp)]
        L.cfi_gguf_type_bytes.argtypes = [C.c_uint32, u64]
        L.cfi_gguf_type_bytes.restype = u64
        L._gguf_ready = True
    return L


class GGUFError(RuntimeError):
    pass


class GGUFFile:
    """A mapped GGUF file: metadata by key, tensors by name (numpy uint8 views of the block bytes)."""

    def __init__(self, path):
        L = _lib()
        h, why = C.c_void_p(), C.create_string_buffer(256)
        if L.cfi_gguf_open(str(path).encode(), C.byref(h), why, 256) != 0:
            raise GGUFError(why.value.decode())
        self.h = h
        self.version = L.cfi_gguf_version(h)
        self.alignment = L.cfi_gguf_alignment(h)

    def close(self):
        if self.h:
            _lib().cfi_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- metadata ----
    def keys(self):
        L = _lib()
        return [L.cfi_gguf_key(self.h, i).decode() for i in range(L.cfi_gguf_kv_count(self.h))]

    def _value(self, i, j, t):
        L = _lib()
        if t == STRING:
            s, n = C.c_char_p(), C.c_uint64()
            if L.cfi_gguf_get_str(self.h, i, j, C.byref(s), C.byref(n)) != 0:
                raise GGUFError("bad string value")
            return C.string_at(s, n.value).decode("utf-8", "replace")
        if t in (F32, F64):
            d = C.c_double()
            L.cfi_gguf_get_f64(self.h, i, j, C.byref(d))
            return d.value
        v = C.c_int64()
        if L.cfi_gguf_get_i64(self.h, i, j, C.byref(v)) != 0:
            raise GGUFError("bad integer value")
        return bool(v.value) if t == BOOL else v.value

    def get(self, key, default=None):
        L = _lib()
        i = L.cfi_gguf_find_key(self.h, key.encode())
        if i < 0:
            return default
        et, n = C.c_int(), C.c_uint64()
        t = L.cfi_gguf_kv_type(self.h, i, C.byref(et), C.byref(n))
        if t == ARRAY:
            if et.value == ARRAY:
                raise GGUFError("nested arrays are not read: " + key)
            return [self._value(i, j, et.value) for j in range(n.value)]
        return self._value(i, 0, t)

    # ---- tensors ----
    def tensor_names(self):
        return [self.info(i)[0] for i in range(_lib().cfi_gguf_tensor_count(self.h))]

    def info(self, i):
        L = _lib()
        name, ty, nd = C.c_char_p(), C.c_uint32(), C.c_uint32()
        dims, nb, data = (C.c_uint64 * 4)(), C.c_uint64(), C.c_void_p()
        if L.cfi_gguf_tensor_info(self.h, i, C.byref(name), C.byref(ty), C.byref(nd), dims, C.byref(nb), C.byref(data)) != 0:
            raise GGUFError("no tensor %d" % i)
        return name.value.decode(), ty.value, tuple(dims[:nd.value]), nb.value, data.value

    def tensor(self, name):
        """(ggml type, dims with ne[0] innermost, numpy uint8 view of the data)."""
        i = _lib().cfi_gguf_find_tensor(self.h, name.encode())
        if i < 0:
            raise KeyError(name)
        _, ty, dims, nb, ptr = self.info(i)
        if nb == 0:
            raise GGUFError("%s: ggml type %d has no known block size" % (name, ty))
        buf = (C.c_uint8 * nb).from_address(ptr)
        return ty, dims, np.frombuffer(buf, dtype=np.uint8)


def _pack_str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _pack_value(t, v):
    if t == STRING:
        return _pack_str(v)
    if t == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_pack_value(et, x) for x in items)
    return struct.pack(_SCALAR[t], v)


def write_gguf(path, kv, tensors, alignment=32):
    """kv: {key: (type, value)} (arrays: (ARRAY, (elem_type, [values]))); tensors: list of
    (name, ggml_type, dims with ne[0] innermost, bytes-like data in ggml's layout)."""
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kv) + (0 if alignment == 32 else 1))
    meta = b"".join(_pack_str(k) + struct.pack("<I", t) + _pack_value(t, v) for k, (t, v) in kv.items())
    if alignment != 32:
        meta += _pack_str("general.alignment") + struct.pack("<II", U32, alignment)
    infos, blobs, off = b"", [], 0
    for name, ty, dims, data in tensors:
        data = bytes(data)
        nbytes = _lib().cfi_gguf_type_bytes(ty, int(np.prod(dims)))
        if nbytes != len(data):
            raise ValueError("%s: %d bytes given, %d expected" % (name, len(data), nbytes))
        infos += _pack_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ty, off)
        blobs.append((off, data))
        off = (off + len(data) + alignment - 1) // alignment * alignment
    body = head + meta + infos
    pad = (-len(body)) % alignment
    with open(path, "wb") as f:
        f.write(body + b"\0" * pad)
        pos = 0
        for o, data in blobs:
            f.write(b"\0" * (o - pos))
            f.write(data)
            pos = o + len(data)
        f.write(b"\0" * ((-pos) % alignment))
