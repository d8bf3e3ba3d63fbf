"""Minimal GGUF tensor reader for the tests (numpy views of a file)."""
import struct

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?",
           10: "<Q", 11: "<q", 12: "<d"}


def read_gguf(path):
    """Returns (kv dict, {name: (ggml_type, dims, bytes)})."""
    buf = open(path, "rb").read()
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from(fmt, buf, off)[0]
        off += struct.calcsize(fmt)
        return v

    def string():
        nonlocal off
        n = take("<Q")
        s = buf[off:off + n].decode()
        off += n
        return s

    def value(t):
        if t == 8:
            return string()
        if t == 9:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        return take(_SCALAR[t])

    assert buf[:4] == b"GGUF"
    off = 4
    _ver, nt, nkv = take("<I"), take("<Q"), take("<Q")
    kv = {}
    for _ in range(nkv):
        k = string()
        kv[k] = value(take("<I"))
    infos = []
    for _ in range(nt):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        infos.append((name, dims, take("<I"), take("<Q")))
    align = kv.get("general.alignment", 32)
    data = (off + align - 1) // align * align
    out = {}
    for name, dims, ty, toff in infos:
        n = int(np.prod(dims))
        nbytes = n * 4 if ty == 0 else n * 2 if ty == 1 else n // 256 * 144 if ty == 12 else 0
        out[name] = (ty, dims, np.frombuffer(buf, np.uint8, nbytes, data + toff))
    return kv, out
