"""The C restatement (oracle/) against the reference library built from its own
sources (oracle/_ref), on models the reference's tests never cover: GQA with
Q4_K weights, multi-step greedy decode, and synthetic files from the product's
GGUF writer.  Also checks the writer's determinism and that the reference
loader accepts its files.
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import golden

Pf = C.POINTER(C.c_float)


def ref_decode(reference, path, tokens):
    """tokens [n_seq, n_steps] -> logits [n_seq, n_steps, V] via reference sessions."""
    g, m = reference.open(path)
    V = reference.config(m)["vocab"]
    out = np.zeros(tokens.shape + (V,), np.float32)
    for i, row in enumerate(tokens):
        s = reference.lib.slate_llama_session_new(m)
        for t, tok in enumerate(row):
            rc = reference.lib.slate_llama_decode_step(s, int(tok), out[i, t].ctypes.data_as(Pf))
            assert rc == 0
        reference.lib.slate_llama_session_free(s)
    reference.close(g, m)
    return out


SYNTH = {
    # BASELINE config 1 shape (all f32, GQA 4/2, hd 16, FFN 172)
    "tiny_f32": dict(n_layers=2, d_model=64, ffn_hidden=172, n_heads=4, n_kv_heads=2, vocab=256,
                     max_seq=128, q4k=False, seed=0),
    # small GQA Q4_K model (group 4, hd 64)
    "gqa_q4k": dict(n_layers=2, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2, vocab=512,
                    max_seq=256, q4k=True, seed=7),
}


@pytest.fixture(scope="module")
def synth_models(sb, workdir):
    paths = {}
    for name, cfg in SYNTH.items():
        p = os.path.join(str(workdir), f"{name}.gguf")
        sb.synth_gguf(p, **cfg)
        paths[name] = p
    return paths


def test_synth_writer_deterministic_across_threads(sb, workdir):
    a, b = os.path.join(str(workdir), "a.gguf"), os.path.join(str(workdir), "b.gguf")
    cfg = dict(SYNTH["gqa_q4k"])
    sb.synth_gguf(a, n_threads=1, **cfg)
    sb.synth_gguf(b, n_threads=5, **cfg)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_synth_layer_period_repeats_layers(sb, workdir):
    """layer_period p: layer l's tensors are byte copies of layer l % p; the
    first p layers and the non-layer tensors are what p = 0 writes."""
    from gguf_util import read_gguf
    cfg = dict(SYNTH["gqa_q4k"], n_layers=5)
    a, b = os.path.join(str(workdir), "p0.gguf"), os.path.join(str(workdir), "p2.gguf")
    sb.synth_gguf(a, **cfg)
    sb.synth_gguf(b, layer_period=2, n_threads=3, **cfg)
    _, ta = read_gguf(a)
    _, tb = read_gguf(b)
    assert ta.keys() == tb.keys()
    for name, (ty, dims, data) in tb.items():
        if name.startswith("blk."):
            l = int(name.split(".")[1])
            src = name.replace(f"blk.{l}.", f"blk.{l % 2}.", 1)
            assert np.array_equal(data, ta[src][2]), name
        else:
            assert np.array_equal(data, ta[name][2]), name
    assert not np.array_equal(ta["blk.2.attn_q.weight"][2], ta["blk.0.attn_q.weight"][2])


def test_synth_weights_statistics(sb, synth_models):
    from gguf_util import read_gguf
    kv, t = read_gguf(synth_models["tiny_f32"])
    assert kv["llama.attention.head_count_kv"] == 2 and kv["llama.vocab_size"] == 256
    emb = t["token_embd.weight"][2].view(np.float32)
    assert abs(emb.mean()) < 2e-3 and abs(emb.std() - 0.02) < 1e-3
    assert np.all(t["blk.0.attn_norm.weight"][2].view(np.float32) == 1.0)


@pytest.mark.parametrize("name", list(SYNTH))
def test_oracle_matches_reference_multistep(oracle, reference, synth_models, name):
    path = synth_models[name]
    rng = np.random.default_rng(3)
    V = SYNTH[name]["vocab"]
    tokens = rng.integers(0, V, size=(3, 12)).astype(np.int32)
    want = ref_decode(reference, path, tokens)
    m = oracle.open(path)
    got, ids = m.decode_many(tokens)
    m.close()
    scale = np.abs(want).max()
    assert np.max(np.abs(got - want)) <= 1e-5 * max(scale, 1.0)
    assert np.array_equal(ids, want.argmax(-1))


@pytest.mark.parametrize("gguf", ["slate_tiny_llama.gguf", "slate_tiny_llama_gqa.gguf",
                                  "slate_tiny_llama_q4k.gguf"])
def test_oracle_matches_reference_on_fixtures(oracle, reference, gguf):
    tokens = np.array([[1, 7, 13, 25, 3, 60, 2, 9], [5, 5, 5, 5, 0, 63, 31, 17]], np.int32)
    want = ref_decode(reference, golden(gguf), tokens)
    m = oracle.open(golden(gguf))
    got, _ = m.decode_many(tokens)
    m.close()
    assert np.max(np.abs(got - want)) <= 1e-5 * max(np.abs(want).max(), 1.0)


def test_oracle_q4k_dot_matches_reference(oracle, reference, sb):
    rng = np.random.default_rng(11)
    w = rng.normal(0, 0.05, (32, 1024)).astype(np.float32)
    q = sb.quantize_q4k(w)
    x = rng.normal(0, 1, 1024).astype(np.float32)
    y_ref = np.zeros(32, np.float32)
    reference.lib.slate_q4_k_matvec(y_ref.ctypes.data_as(Pf), q.ctypes.data, x.ctypes.data_as(Pf), 32, 1024)
    y = oracle.q4k_matvec(q, x, 32, 1024)
    assert np.max(np.abs(y - y_ref)) <= 1e-5 * np.abs(y_ref).max()


def test_reference_cuda_stub_is_null(reference):
    """backend_cuda_stub.c:33 -- the reference's own stub stays NULL, so its CPU
    path (the oracle) never reaches a GPU."""
    assert not reference.lib.slate_backend_cuda()
    assert reference.lib.slate_backend_default() == reference.lib.slate_backend_cpu()
