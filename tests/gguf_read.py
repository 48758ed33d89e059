"""Minimal pure-Python GGUF reader for tests (independent of both the product and the oracle)."""
import struct

import numpy as np

_SS = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}


def _str(b, o):
    n = struct.unpack_from("<Q", b, o)[0]
    return b[o + 8:o + 8 + n].decode(), o + 8 + n


def read_header(path):
    b = open(path, "rb").read()
    magic, ver, nt, nkv = struct.unpack_from("<IIQQ", b, 0)
    assert magic == 0x46554747 and ver in (2, 3)
    o = 24
    kv = {}
    for _ in range(nkv):
        k, o = _str(b, o)
        ty = struct.unpack_from("<I", b, o)[0]
        o += 4
        if ty == 8:
            v, o = _str(b, o)
        elif ty == 9:
            et, n = struct.unpack_from("<IQ", b, o)
            o += 12
            v = []
            for _ in range(n):
                if et == 8:
                    s, o = _str(b, o)
                    v.append(s)
                else:
                    o += _SS[et]
        else:
            fmt = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}[ty]
            v = struct.unpack_from("<" + fmt, b, o)[0]
            o += _SS[ty]
        kv[k] = v
    tensors = {}
    for _ in range(nt):
        name, o = _str(b, o)
        nd = struct.unpack_from("<I", b, o)[0]
        o += 4
        ne = list(struct.unpack_from("<" + "Q" * nd, b, o))
        o += 8 * nd
        ty, off = struct.unpack_from("<IQ", b, o)
        o += 12
        tensors[name] = (ne, ty, off)
    align = kv.get("general.alignment", 32)
    data = (o + align - 1) // align * align
    return b, kv, tensors, data


def read_tensor(path, name, n=None):
    b, kv, tensors, data = read_header(path)
    ne, ty, off = tensors[name]
    dt = {0: np.float32, 1: np.uint16, 30: np.uint16}[ty]
    count = int(np.prod(ne)) if n is None else n
    return np.frombuffer(b, dt, count, data + off).copy()


def _f16_flush(u16):
    """f16 bits -> f32 as the reference's to_f32 reads them (subnormals flushed, src/gguf.cpp:201-212)."""
    u = u16.astype(np.uint32)
    sign, exp, man = (u >> 15) & 1, (u >> 10) & 0x1F, u & 0x3FF
    bits = np.where(exp == 0, sign << 31,
                    np.where(exp == 31, (sign << 31) | 0x7F800000 | (man << 13), (sign << 31) | ((exp + 112) << 23) | (man << 13)))
    return bits.astype(np.uint32).view(np.float32)


def tensor_f32(b, tensors, data, name):
    """A tensor's values as f32 exactly as to_f32 (src/gguf.cpp:193-234) gives them, and its type."""
    ne, ty, off = tensors[name]
    n = int(np.prod(ne))
    if ty == 0:
        v = np.frombuffer(b, np.float32, n, data + off).copy()
    elif ty == 1:
        v = _f16_flush(np.frombuffer(b, np.uint16, n, data + off))
    elif ty == 30:
        v = (np.frombuffer(b, np.uint16, n, data + off).astype(np.uint32) << 16).view(np.float32)
    elif ty == 8:
        blk = np.frombuffer(b, np.uint8, n // 32 * 34, data + off).reshape(-1, 34)
        s = _f16_flush(blk[:, :2].copy().view(np.uint16)[:, 0])
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        v = (s[:, None] * q).reshape(-1).astype(np.float32)
    else:
        raise ValueError(f"type {ty}")
    return v, ty


def device_weights(path):
    """W(name) -> float64 numpy of the values the reference's device holds after
    WeightSet::load(keep_f32) (src/net.mm:126-173): f32 tensors as stored, every other type rounded
    to f16 (round to nearest even; the reference truncates f16 subnormals, below 6.1e-5), shaped
    [ne1, ne0] for matrices. Also returns the KV dict."""
    b, kv, tensors, data = read_header(path)

    def W(name, host=False):   # host: the to_f32 values the reference's host copies hold (embeddings)
        ne, ty, off = tensors[name]
        v, ty = tensor_f32(b, tensors, data, name)
        if ty != 0 and not host:
            v = v.astype(np.float16).astype(np.float32)
        v = v.astype(np.float64)
        return v.reshape(ne[::-1]) if len(ne) > 1 else v
    return W, kv
