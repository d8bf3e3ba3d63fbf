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


def _q4k_dequant_ggml(raw, n_blocks):
    """llama.cpp / ggml's Q4_K element order (restated from ggml's
    dequantize_row_q4_k): for the 64-element pair g, element e of sub-block 2g
    is the low nibble of qs[32g + e] and of 2g + 1 the high nibble; the header
    (d, dmin, packed 6-bit scales / mins) is as in util/quant.c:139-166."""
    b = raw.reshape(n_blocks, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dm = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    sc_b = b[:, 4:16].astype(np.int32)
    sc = np.zeros((n_blocks, 8), np.int32)
    mn = np.zeros((n_blocks, 8), np.int32)
    for j in range(8):
        if j < 4:
            sc[:, j] = sc_b[:, j] & 63
            mn[:, j] = sc_b[:, j + 4] & 63
        else:
            sc[:, j] = (sc_b[:, j + 4] & 15) | ((sc_b[:, j - 4] >> 6) << 4)
            mn[:, j] = (sc_b[:, j + 4] >> 4) | ((sc_b[:, j] >> 6) << 4)
    qs = b[:, 16:].astype(np.int32)
    out = np.zeros((n_blocks, 256), np.float32)
    for g in range(4):
        q = qs[:, 32 * g:32 * g + 32]
        for half, s in ((0, 2 * g), (1, 2 * g + 1)):
            nib = (q >> 4) if half else (q & 15)
            out[:, 32 * s:32 * s + 32] = (d * sc[:, s])[:, None] * nib - (dm * mn[:, s])[:, None]
    return out.reshape(-1)


def test_synth_llama_cpp_order_and_f16_tables(sb, oracle, workdir):
    """q4k_order=1 writes the same weights in llama.cpp's nibble order (each
    Q4_K tensor decodes under ggml's rules to what the Slate-order file decodes
    to under Slate's); embd_f16=1 stores the embedding table as f16 with the
    values that embd_f16=2 stores as f32."""
    from gguf_util import read_gguf
    cfg = dict(SYNTH["gqa_q4k"])
    paths = {}
    for name, kw in (("s", {}), ("g", {"q4k_order": 1}), ("h", {"embd_f16": 1}),
                     ("r", {"embd_f16": 2})):
        paths[name] = os.path.join(str(workdir), f"order_{name}.gguf")
        sb.synth_gguf(paths[name], **cfg, **kw)
    _, ts = read_gguf(paths["s"])
    _, tg = read_gguf(paths["g"])
    n_q4k = 0
    for name, (ty, dims, data) in ts.items():
        if ty != 12:
            assert np.array_equal(data, tg[name][2]), name
            continue
        n_q4k += 1
        nb = len(data) // 144
        want = oracle.dequant_q4k(data, nb * 256)
        got = _q4k_dequant_ggml(tg[name][2], nb)
        assert np.array_equal(got, want), name
        assert not np.array_equal(data, tg[name][2])
    assert n_q4k > 0
    _, th = read_gguf(paths["h"])
    _, tr = read_gguf(paths["r"])
    assert th["token_embd.weight"][0] == 1 and tr["token_embd.weight"][0] == 0
    assert np.array_equal(th["token_embd.weight"][2].view(np.float16).astype(np.float32),
                          tr["token_embd.weight"][2].view(np.float32))


def test_cpu_writer_matches_product_writer(sb, workdir):
    """oracle.synth_gguf (synth.c built without CUDA, used where the reference is
    timed) writes the same bytes as the product library's writer."""
    import oracle as O
    a, b = os.path.join(str(workdir), "w_oracle.gguf"), os.path.join(str(workdir), "w_product.gguf")
    for cfg in (SYNTH["gqa_q4k"], dict(SYNTH["tiny_f32"], embd_f16=2)):
        O.synth_gguf(a, **cfg)
        sb.synth_gguf(b, **cfg)
        assert open(a, "rb").read() == open(b, "rb").read()


def test_reference_seeded_history_matches_engine_generator(reference, oracle, synth_models):
    """slate_ref_session_seed_context (oracle/ref_session.c) gives a reference
    session the history the CUDA engine's seed_context writes: a session seeded
    that way decodes like an oracle session given the generator's K/V."""
    from gpu_util import seeded_kv
    path = synth_models["gqa_q4k"]
    g, m = reference.open(path)
    c = reference.config(m)
    kvd = c["n_kv_heads"] * c["head_dim"]
    n, seed, tok = 37, 4242, 11
    s = reference.session(m, n, seed)
    assert reference.lib.slate_llama_session_position(s) == n
    got = np.zeros(c["vocab"], np.float32)
    assert reference.decode(s, tok, got) == 0
    reference.lib.slate_llama_session_free(s)
    reference.close(g, m)
    om = oracle.open(path)
    o = om.session()
    K, V = seeded_kv(seed, n, c["n_layers"], kvd)
    assert o.seed_kv(K, V) == 0
    rc, want = o.decode(tok)
    assert rc == 0
    o.close()
    om.close()
    assert np.max(np.abs(got - want)) <= 1e-5 * np.abs(want).max()
