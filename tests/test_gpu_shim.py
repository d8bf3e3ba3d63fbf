"""Drop-in check: the engine built from slate's OWN loader.

The reference library (oracle/_ref, slate's unmodified sources) opens the GGUF
with slate_gguf_open + slate_llama_open; the integration shim
(slate_b200/shim/slate_llama_cuda_shim.c, compiled against slate's headers)
turns that slate_llama_t into a device engine; the engine's logits are then
compared with slate_llama_prefill run by the same reference library on the
same model object (tests/test_llama_infer*.c tolerance: Linf < 1e-3)."""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import ROOT, golden
from gpu_util import scale_err
from test_golden import TINY, read_ref_logits

pytestmark = pytest.mark.gpu
SHIM = os.path.join(ROOT, "oracle", "_ref", "libslate_shim.so")


@pytest.mark.parametrize("gguf,ref", TINY)
def test_engine_from_reference_loader(sb, reference, gguf, ref):
    if not os.path.exists(SHIM):
        pytest.skip("integration shim not built (reference headers were unavailable)")
    shim = C.CDLL(SHIM)
    shim.slate_llama_batch_new.restype = C.c_void_p
    shim.slate_llama_batch_new.argtypes = [C.c_void_p, C.POINTER(sb.CudaOpts)]
    prompt, want = read_ref_logits(ref)
    g, m = reference.open(golden(gguf))
    opts = sb.CudaOpts(0, 4, 4, sb.KV_F32, 0, 0, 0, 1, 0)
    h = shim.slate_llama_batch_new(m, C.byref(opts))
    assert h, sb.last_error()
    slot = sb.F["slate_llama_batch_open"](h)
    V = sb.F["slate_llama_batch_vocab"](h)
    got = np.zeros(V, np.float32)
    p = np.ascontiguousarray(prompt)
    rc = sb.F["slate_llama_batch_prefill"](h, slot, p.ctypes.data_as(C.POINTER(C.c_int32)), len(p),
                                           got.ctypes.data_as(C.POINTER(C.c_float)))
    assert rc == 0, sb.last_error()
    # the reference's own CPU path on the same slate_llama_t
    s = reference.lib.slate_llama_session_new(m)
    cpu = np.zeros(V, np.float32)
    assert reference.lib.slate_llama_prefill(s, p.ctypes.data_as(C.POINTER(C.c_int32)), len(p),
                                             cpu.ctypes.data_as(C.POINTER(C.c_float))) == 0
    reference.lib.slate_llama_session_free(s)
    sb.F["slate_llama_batch_free"](h)
    reference.close(g, m)
    assert np.max(np.abs(got - want)) < 1e-3
    assert scale_err(got, cpu) < 1e-4
