"""GPU-test helpers: call the CUDA backend's vtable through its C function
pointers (the same entry points a reference caller would use)."""
import ctypes as C

import numpy as np

p, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t

SIGS = {
    "alloc": (p, sz), "release": (None, p), "copy_h2d": (None, p, p, sz),
    "copy_d2h": (None, p, p, sz), "matvec": (None, p, p, p, i32, i32),
    "linear_batch": (None, p, p, p, i32, i32, i32), "matvec_q4k": (None, p, p, p, i32, i32),
    "rmsnorm_row": (None, p, p, p, i32, f32), "silu_mul": (None, p, p, p, i32),
    "add_inplace": (None, p, p, i32), "embed_lookup": (None, p, p, i32, i32),
    "attention_step": (None, p, p, p, p, p, i32, i32), "sync": (None,),
}
EXT = {
    "matmul_q4k_batch": (i32, p, p, p, i32, i32, i32),
    "matmul_f32_batch": (i32, p, p, p, i32, i32, i32),
    "rmsnorm_rows": (i32, p, p, p, i32, i32, f32),
    "argmax_rows": (i32, p, p, i32, i32),
    "rope_kv_append_paged": (i32, p, p, p, p, p, p, i32, p, i64, i32, i32, i32, i32, i32, i32, p, p),
    "attention_paged_gqa": (i32, p, p, p, p, p, i32, p, i64, i32, i32, i32, i32, i32, i32),
    "matmul_q4k_batch_tc": (i32, p, p, p, i32, i32, i32, i32),
}


class Backend:
    def __init__(self, sb, device=0):
        ptr = sb.F["slate_backend_cuda_create"](device)
        if not ptr:
            raise RuntimeError(sb.last_error())
        self.sb = sb
        s = ptr.contents
        self.name = s.base.name.decode()
        self.fn = {}
        for n, sig in SIGS.items():
            self.fn[n] = C.CFUNCTYPE(*sig)(getattr(s.base, n))
        for n, sig in EXT.items():
            self.fn[n] = C.CFUNCTYPE(*sig)(getattr(s, n))
        self.live = []

    def __getattr__(self, n):
        return self.fn[n]

    def dev(self, a):
        a = np.ascontiguousarray(a)
        d = self.fn["alloc"](max(a.nbytes, 4))
        assert d
        if a.nbytes:
            self.fn["copy_h2d"](d, a.ctypes.data, a.nbytes)
        self.live.append(d)
        return d

    def empty(self, nbytes):
        d = self.fn["alloc"](max(nbytes, 4))
        assert d
        self.live.append(d)
        return d

    def host(self, d, shape, dtype=np.float32):
        out = np.zeros(shape, dtype)
        self.fn["sync"]()
        self.fn["copy_d2h"](out.ctypes.data, d, out.nbytes)
        return out

    def free_all(self):
        for d in self.live:
            self.fn["release"](d)
        self.live = []


def seeded_kv(seed, n, n_layers, kv_dim):
    """The history slate_llama_batch_seed_context writes for `seed`: element i of
    the [layer][K|V][token][kv_dim] order is 2*u - 1 in f32, u the top 53 bits of
    splitmix64(seed ^ i * 0x9e3779b97f4a7c15) scaled to [0, 1).  Returns
    (K, V), each [n_layers, n, kv_dim] f32."""
    with np.errstate(over="ignore"):
        i = np.arange(n_layers * 2 * n * kv_dim, dtype=np.uint64)
        z = np.uint64(seed) ^ (i * np.uint64(0x9E3779B97F4A7C15))
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = ((z >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)).astype(np.float32)
    kv = (u * np.float32(2.0) - np.float32(1.0)).reshape(n_layers, 2, n, kv_dim)
    return np.ascontiguousarray(kv[:, 0]), np.ascontiguousarray(kv[:, 1])


def scale_err(got, want):
    """max |got - want| relative to the reference's largest magnitude."""
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / max(np.abs(want).max(), 1e-30))


def greedy_agrees(engine_id, ref_logits, tol_abs):
    """Exact match, or a near-tie: the reference's top-2 gap is below tol_abs and
    the engine picked one of the tied candidates."""
    top = int(np.argmax(ref_logits))
    if engine_id == top:
        return True, False
    gap = ref_logits[top] - ref_logits[engine_id]
    return bool(gap <= tol_abs), True
