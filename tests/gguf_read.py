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
