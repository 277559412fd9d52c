"""The C oracle against the independent numpy restatement (tests/numpy_ref.py) and the invariants the
reference's own tests hold (prefix forward equals full forward, `tests/engine_parity.rs:59-85`).
These pin the oracle before it is used to judge the CUDA path."""
import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M


def test_f16_conversion_matches_ieee():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, 200_000, dtype=np.uint64).astype(np.uint32)
    xs = bits.view(np.float32)
    xs = xs[np.isfinite(xs)]
    special = np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.0**-24, 2.0**-25, 3 * 2.0**-26, 2.0**-14,
                        2.0**-14 - 2.0**-25, 1.0 + 2.0**-11, 1.0 + 3 * 2.0**-11, -5.9604645e-08], np.float32)
    dense = (rng.standard_normal(100_000) * np.exp(rng.uniform(-20, 12, 100_000))).astype(np.float32)
    lib = oracle.lib()
    for x in np.concatenate([xs[:20000], special, dense[:20000]]):
        h = lib.or_f32_to_f16(float(x))
        want = np.array([x], np.float32).astype(np.float16).view(np.uint16)[0]
        assert h == want, (x, hex(h), hex(want))
        if (h & 0x7C00) != 0x7C00:
            assert lib.or_f16_to_f32(h) == np.float32(np.array([h], np.uint16).view(np.float16)[0])


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("m", [1, 7, 20, 21, 64])
def test_matmul_variants(bits, m):
    rng = np.random.default_rng(bits * 100 + m)
    n, k = 128, 512
    packed, scales = M._quant_tensor(rng, n, k, bits, 0.05)
    a = rng.standard_normal((m, k)).astype(np.float16)
    y = oracle.matmul(a, packed, scales, n, k, bits)
    w32 = M.dequant(packed, scales, bits, k)
    tiled = m > 20 and bits == 4
    w = w32.astype(np.float16).astype(np.float32) if tiled else w32
    want = (a.astype(np.float64) @ w.T.astype(np.float64))
    np.testing.assert_allclose(y.astype(np.float64), want, rtol=2e-3, atol=2e-3)
    if tiled:  # the tiled path really dequantizes through f16 (`src/kernels.rs:671`)
        g = oracle.matmul(a, packed, scales, n, k, bits, variant=1)
        assert np.abs(g.astype(np.float32) - y.astype(np.float32)).max() < 5e-3


def test_attention_matches_softmax():
    rng = np.random.default_rng(1)
    hq, hk, hd, l = 8, 2, 256, 300
    q = rng.standard_normal((hq, l, hd)).astype(np.float16)
    k = rng.standard_normal((hk, l, hd)).astype(np.float16)
    v = rng.standard_normal((hk, l, hd)).astype(np.float16)
    gate = rng.standard_normal((l, hq * 2 * hd)).astype(np.float16)
    out = oracle.attn(q, k, v, gate, hq * 2 * hd, hd, 2 * hd)
    qs = (q.astype(np.float32) * np.float32(1 / 16)).astype(np.float16).astype(np.float64)
    mask = np.tril(np.ones((l, l), bool))
    for h in range(hq):
        kh = h // 4
        s = qs[h] @ k[kh].T.astype(np.float64)
        s = np.where(mask, s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        g = gate[:, h * 2 * hd + hd:h * 2 * hd + 2 * hd].astype(np.float64)
        want = (p @ v[kh].astype(np.float64)) / (1 + np.exp(-g))
        np.testing.assert_allclose(out[:, h * hd:(h + 1) * hd].astype(np.float64), want, atol=2e-3, rtol=2e-3)


def test_attention_with_prefix_rows():
    """Queries at positions p.. attend to cached rows 0..p-1 as well (the snapshot continuation)."""
    rng = np.random.default_rng(2)
    hq, hk, hd, p, l = 8, 2, 256, 37, 20
    q = rng.standard_normal((hq, p + l, hd)).astype(np.float16)
    k = rng.standard_normal((hk, p + l, hd)).astype(np.float16)
    v = rng.standard_normal((hk, p + l, hd)).astype(np.float16)
    full = oracle.attn(q, k, v)
    tail = oracle.attn(q[:, p:], k, v, p=p)
    np.testing.assert_allclose(tail.astype(np.float32), full[p:].astype(np.float32), atol=1e-3)


def test_gdn_matches_recurrence():
    rng = np.random.default_rng(3)
    l, h, dk, dv = 50, 4, 128, 128
    q = rng.standard_normal((l, h, dk)).astype(np.float32)
    k = rng.standard_normal((l, h, dk)).astype(np.float32)
    v = rng.standard_normal((l, h, dv)).astype(np.float32)
    beta = 1 / (1 + np.exp(-rng.standard_normal((l, h)))).astype(np.float32)
    decay = np.exp(-np.log1p(np.exp(rng.standard_normal((l, h))))).astype(np.float32)
    s0 = rng.standard_normal((h, dk, dv)).astype(np.float32) * 0.1
    o, st = oracle.gdn(q, k, v, beta, decay, s0)
    S = s0.astype(np.float64)
    for t in range(l):
        qn = q[t] / np.sqrt((q[t].astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6) / np.sqrt(dk)
        kn = k[t] / np.sqrt((k[t].astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)
        S = S * decay[t][:, None, None]
        kv = np.einsum("hkv,hk->hv", S, kn)
        S = S + kn[:, :, None] * ((v[t] - kv) * beta[t][:, None])[:, None, :]
        np.testing.assert_allclose(o[t].reshape(h, dv), np.einsum("hkv,hk->hv", S, qn), atol=2e-4, rtol=1e-4)
    np.testing.assert_allclose(st, S, atol=2e-4, rtol=1e-4)
    # split in two calls with the state carried = one call
    o1, s1 = oracle.gdn(q[:20], k[:20], v[:20], beta[:20], decay[:20], s0)
    o2, s2 = oracle.gdn(q[20:], k[20:], v[20:], beta[20:], decay[20:], s1)
    np.testing.assert_allclose(np.concatenate([o1, o2]), o, atol=1e-5)
    np.testing.assert_allclose(s2, st, atol=1e-5)


def test_decode_scales_matches_numpy():
    rng = np.random.default_rng(4)
    s = (rng.standard_normal((7, 64)) * 0.01).astype(np.float16)
    enc, dec = M.encode_scales_u8(s)
    got = oracle.decode_scales(enc, 7, 64)
    assert np.array_equal(got.view(np.uint16), dec.view(np.uint16))
    # the codes approximate the scales (127 log steps per row span its range)
    np.testing.assert_allclose(got.astype(np.float32), s.astype(np.float32), rtol=3e-2, atol=1e-6)


def test_head_probs_matches_numpy():
    rng = np.random.default_rng(5)
    d, dim = 2048, 256
    head = {"norm.weight": rng.standard_normal(d), "norm.bias": rng.standard_normal(d) * 0.1,
            "q.weight": rng.standard_normal((dim, d)) / 45, "q.bias": rng.standard_normal(dim) * 0.1,
            "k.weight": rng.standard_normal((dim, d)) / 45, "k.bias": rng.standard_normal(dim) * 0.1}
    head = {k: v.astype(np.float32) for k, v in head.items()}
    hidden = rng.standard_normal((4, d)).astype(np.float32)
    p = oracle.head_probs(hidden, head, 0.7)

    def proj(x, w, b):
        x = x.astype(np.float64)
        xn = (x - x.mean()) / np.sqrt(x.var() + 1e-5) * head["norm.weight"] + head["norm.bias"]
        return head[w].astype(np.float64) @ xn + head[b]
    q = proj(hidden[-1], "q.weight", "q.bias")
    logits = np.array([proj(r, "k.weight", "k.bias") @ q for r in hidden[:-1]]) * dim ** -0.5 / 0.7
    e = np.exp(logits - logits.max())
    np.testing.assert_allclose(p, e / e.sum(), rtol=1e-12, atol=1e-14)


def test_engine_matches_numpy_torso(small_model):
    from tests.numpy_ref import NumpyTorso
    e = oracle.Engine(small_model)
    ref = NumpyTorso(small_model)
    rng = np.random.default_rng(6)
    for l in (9, 40):
        ids = rng.integers(0, 8192, l)
        hid, _, tr = e.forward(ids, list(range(l)), trace=True)
        ntr, nh = ref.forward(ids)
        assert np.abs(tr - ntr).max() < 2e-2, np.abs(tr - ntr).max(axis=(1, 2))
        assert np.abs(hid - nh).max() < 2e-2


def test_prefix_forward_matches_full(small_model):
    """`tests/engine_parity.rs:59-85` on the oracle: a question continued from the state's snapshot
    gives the hidden rows of the whole prompt (the short question runs the GEMV path, the whole
    prompt the tiled one, so they differ by f16 dequant rounding only)."""
    e = oracle.Engine(small_model)
    rng = np.random.default_rng(7)
    state = rng.integers(0, 8000, 70)
    _, snap, _ = e.forward(state, [], keep=True)
    assert snap.len == 70
    for ql in (12, 33):
        q = rng.integers(0, 8000, ql)
        rows = [3, ql - 1]
        a, _, _ = e.forward(q, rows, cache=snap)
        b, _, _ = e.forward(np.concatenate([state, q]), [70 + r for r in rows])
        assert np.abs(a - b).max() < (2e-2 if ql <= 20 else 1e-6)
    # a snapshot of a snapshot continuation covers both parts
    _, snap2, _ = e.forward(q, [], cache=snap, keep=True)
    assert snap2.len == 70 + 33


def test_engine_rejects_bad_input(small_model):
    e = oracle.Engine(small_model)
    with pytest.raises(ValueError):
        e.forward([1, 2, 3], [3])
    with pytest.raises(ValueError):
        e.forward([], [])
    with pytest.raises(ValueError):
        e.forward(np.zeros(4097, np.int64), [])


def test_u8_embedding_and_adapter_layers(small_model_u8, adapter_model):
    from tests.numpy_ref import NumpyTorso
    for path, vocab in ((small_model_u8, 8192), (adapter_model, 4096)):
        e = oracle.Engine(path)
        ref = NumpyTorso(path)
        ids = np.random.default_rng(8).integers(0, vocab, 25)
        _, _, tr = e.forward(ids, [], trace=True)
        ntr, _ = ref.forward(ids)
        assert np.abs(tr - ntr).max() < 2e-2
