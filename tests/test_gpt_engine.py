"""The reference's GPT-style inference engine (src/infer/engine.c), unchanged,
on this library's CUDA vtable.

That engine is the one the reference's scheduler and server drive
(src/server/scheduler.c:47,78).  It uses its backend with the CPU backend's
semantics: host memset / memcpy on buffers from alloc (engine.c:276-277,
411-412, 586-591), host weight, scratch and logits pointers passed to the
entries, results read without sync().  slate_backend_cuda_host_coherent serves
it as is.  oracle/_ref/libslate_gpt_drive.so (tests/gpt_engine_drive.c) builds
the reference's causal LM and runs prefill plus teacher-forced
slate_infer_batch_step calls on a given backend; the GPU test compares every
logit with the reference's CPU backend within 1e-4 of the logit scale (the
vtable's conformance bound, as in test_backend.c).
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import ROOT

DRIVE = os.path.join(ROOT, "oracle", "_ref", "libslate_gpt_drive.so")
CFG = dict(vocab=256, max_seq=64, d_model=64, n_layers=2, ffn_hidden=128, n_seq=4, prompt_len=5,
           steps=6)


def drive(backend, relocate):
    if not os.path.exists(DRIVE):
        pytest.skip("oracle/_ref/libslate_gpt_drive.so not built (reference headers unavailable)")
    lib = C.CDLL(DRIVE)
    lib.gpt_engine_drive.restype = C.c_int
    lib.gpt_engine_drive.argtypes = [C.c_void_p] + [C.c_int] * 9 + [C.c_void_p]
    c = CFG
    out = np.zeros((1 + c["steps"], c["n_seq"], c["vocab"]), np.float32)
    rc = lib.gpt_engine_drive(backend, c["vocab"], c["max_seq"], c["d_model"], c["n_layers"],
                              c["ffn_hidden"], c["n_seq"], c["prompt_len"], c["steps"],
                              int(relocate), out.ctypes.data)
    return rc, out


def test_gpt_engine_drive_on_reference_cpu_backend():
    for relocate in (0, 1):
        rc, a = drive(None, relocate)
        assert rc == 0
        assert np.isfinite(a).all() and np.abs(a).max() > 0
        rc, b = drive(None, relocate)
        assert rc == 0 and np.array_equal(a, b)
    # the model moved onto the backend runs the same computation
    assert np.max(np.abs(drive(None, 1)[1] - a)) <= 1e-5 * np.abs(a).max()


def _compare(got, want):
    for i in range(want.shape[0]):          # the prompt block, then each batch step
        scale = float(np.abs(want[i]).max())
        err = float(np.max(np.abs(got[i].astype(np.float64) - want[i]))) / scale
        assert err <= 1e-4, (i, err)
        assert (np.argmax(got[i], axis=1) == np.argmax(want[i], axis=1)).all()


@pytest.mark.gpu
def test_gpt_engine_on_cuda_vtable(sb):
    """The model moved onto the backend (its parameters in alloc'd memory) and
    the prompts through slate_infer_batch_step: the engine hands the CUDA table
    only memory that table allocated."""
    be = sb.F["slate_backend_cuda_host_coherent"](0)
    assert be, sb.last_error()
    rc, want = drive(None, 1)
    assert rc == 0
    rc, got = drive(be, 1)
    assert rc == 0, sb.last_error()
    _compare(got, want)


@pytest.mark.gpu
def test_gpt_engine_host_pointers_on_cuda_vtable(sb):
    """The engine exactly as the reference's callers use it -- weights in the
    module's host arena, slate_infer_prefill with its host scratch -- where the
    device reads pageable host memory."""
    if sb.F["slate_cuda_pageable_memory_access"](0) != 1:
        pytest.skip("the device cannot read pageable host memory (no HMM / ATS)")
    be = sb.F["slate_backend_cuda_host_coherent"](0)
    assert be, sb.last_error()
    rc, want = drive(None, 0)
    assert rc == 0
    rc, got = drive(be, 0)
    assert rc == 0, sb.last_error()
    _compare(got, want)
