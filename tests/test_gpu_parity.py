"""The CUDA path through the C ABI against the CPU oracle, on the same seeded inputs.

Tolerances (from the build's parity targets): per-layer hidden states within 2e-2 max-abs; answer
probabilities within 1e-3 with identical argmax; single kernels as stated per test (f16 outputs:
a few f16 ulps; f32 recurrences: 1e-4 relative)."""
import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("m", [1, 7, 33, 100, 130, 300, 700])
@pytest.mark.parametrize("n,k", [(8256, 2048), (2048, 6144), (384, 192)])  # 192: an odd k-tile count
def test_matmul_matches_oracle(torch, m, n, k):
    from strands_decider.engine import QWeight
    rng = np.random.default_rng(m * 7 + n)
    packed, scales = M._quant_tensor(rng, n, k, 4, 1.0 / np.sqrt(k))
    a = rng.standard_normal((m, k)).astype(np.float16)
    want = oracle.matmul(a, packed, scales, n, k, 4, variant=2).astype(np.float32)  # f16 dequant, f32 acc
    q_d, s_d, a_d = dev(torch, packed), dev(torch, scales.view(np.uint16)), dev(torch, a.view(np.uint16))
    w = QWeight(q_d.data_ptr(), s_d.data_ptr(), n, k)
    y = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    ws = torch.zeros(16 << 20, dtype=torch.float32, device="cuda")
    for ws_bytes in (0, ws.numel() * 4):  # without and with split-K
        y.zero_()
        w.matmul(a_d.data_ptr(), m, y.data_ptr(), n, ws_dev=ws.data_ptr(), ws_bytes=ws_bytes)
        torch.cuda.synchronize()
        got = y.cpu().numpy().astype(np.float32)
        err = np.abs(got - want)
        assert err.max() <= 2e-3 + 2e-3 * np.abs(want).max(), (ws_bytes, err.max())


@pytest.mark.parametrize("m", [1, 8, 9, 33, 64, 100, 128, 256])
@pytest.mark.parametrize("n,k", [(8256, 2048), (2048, 6144), (384, 256)])
def test_matmul_small_m_kernel(torch, m, n, k):
    """The small-M kernel (sd_matmul_ex algo 2: mma.sync on weights dequantized in registers, K split over
    a cluster) against the oracle's f16-dequant matmul and against the tcgen05 tiles (algo 1); the
    planner's choice (algo 0) is one of the two, bit for bit (the small-M kernel up to 16 tokens, and up
    to 64 for outputs of at most 4096); two runs agree bit for bit (the cluster adds its splits in rank
    order). Shapes: in_proj, down (the deepest K split), and a short K with a ragged 128-row block."""
    from strands_decider.engine import QWeight
    rng = np.random.default_rng(m * 11 + n + k)
    packed, scales = M._quant_tensor(rng, n, k, 4, 1.0 / np.sqrt(k))
    a = rng.standard_normal((m, k)).astype(np.float16)
    want = oracle.matmul(a, packed, scales, n, k, 4, variant=2).astype(np.float32)
    q_d, s_d, a_d = dev(torch, packed), dev(torch, scales.view(np.uint16)), dev(torch, a.view(np.uint16))
    w = QWeight(q_d.data_ptr(), s_d.data_ptr(), n, k)
    ws = torch.zeros(16 << 20, dtype=torch.float32, device="cuda")
    outs = {}
    for algo in (2, 2, 1, 0):
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        w.matmul_ex(a_d.data_ptr(), m, y.data_ptr(), n, ws_dev=ws.data_ptr(), ws_bytes=ws.numel() * 4, algo=algo)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        if algo == 2 and 2 in outs:
            assert np.array_equal(got.view(np.uint16), outs[2].view(np.uint16))
        outs[algo] = got
    small = outs[2].astype(np.float32)
    assert np.isfinite(small).all()
    tol = 2e-3 + 2e-3 * np.abs(want).max()
    assert np.abs(small - want).max() <= tol
    assert np.abs(small - outs[1].astype(np.float32)).max() <= tol
    pick = 2 if (m <= 16 or (m <= 64 and n <= 4096)) else 1
    assert np.array_equal(outs[0].view(np.uint16), outs[pick].view(np.uint16))


@pytest.mark.parametrize("m", [5, 40, 128, 200])
@pytest.mark.parametrize("epi", ["silu", "add"])
def test_matmul_small_m_epilogues(torch, m, epi):
    """The small-M kernel's other epilogues: SwiGLU of interleaved gate/up rows, and the f16-rounded
    products added into f32 residual rows (x += f16(a W^T), `add_norm`'s add, src/kernels.rs:93-120),
    against the oracle and against the tcgen05 tiles."""
    from strands_decider.engine import QWeight
    n, k = 2048, 2048
    rng = np.random.default_rng(m + (epi == "add"))
    packed, scales = M._quant_tensor(rng, n, k, 4, 1.0 / np.sqrt(k))
    a = rng.standard_normal((m, k)).astype(np.float16)
    want = oracle.matmul(a, packed, scales, n, k, 4, variant=2).astype(np.float32)
    q_d, s_d, a_d = dev(torch, packed), dev(torch, scales.view(np.uint16)), dev(torch, a.view(np.uint16))
    silu = epi == "silu"
    w = QWeight(q_d.data_ptr(), s_d.data_ptr(), n, k, interleave=silu)
    got = {}
    if silu:
        g, u = want[:, :n // 2], want[:, n // 2:]
        g, u = g.astype(np.float16).astype(np.float32), u.astype(np.float16).astype(np.float32)
        want = g / (1 + np.exp(-g)) * u
        for algo in (1, 2):
            y = torch.full((m, n // 2), float("nan"), dtype=torch.float16, device="cuda")
            w.matmul_ex(a_d.data_ptr(), m, y.data_ptr(), n // 2, silu=True, algo=algo)
            torch.cuda.synchronize()
            got[algo] = y.cpu().numpy().astype(np.float32)
        tol = 4e-3 * (1 + np.abs(want).max())
    else:
        x0 = rng.standard_normal((m, n)).astype(np.float32)
        want = x0 + want.astype(np.float16).astype(np.float32)
        for algo in (1, 2):
            x = dev(torch, x0)
            w.matmul_ex(a_d.data_ptr(), m, None, n, x_dev=x.data_ptr(), algo=algo)
            torch.cuda.synchronize()
            got[algo] = x.cpu().numpy()
        tol = 2e-3 + 2e-3 * np.abs(want).max()
    assert np.isfinite(got[2]).all()
    assert np.abs(got[2] - want).max() <= tol
    assert np.abs(got[2] - got[1]).max() <= tol


@pytest.mark.parametrize("bits,group,asym", [(3, 32, False), (2, 32, False), (4, 64, False), (3, 128, False), (2, 256, False),
                                             (4, 32, True), (3, 64, True), (2, 128, True)])
@pytest.mark.parametrize("m", [5, 300])
def test_matmul_other_formats_match_oracle(torch, bits, group, asym, m):
    """The reference's other weight formats (int3 and int2 codes, groups of 64-256 weights per scale,
    asymmetric weights q * scale + bias with an f16 bias per group), which it serves through its GEMV
    with f32 dequantization (`src/engine.rs:432-441`, `src/kernels.rs:545-635`): repacked into the int4
    tile layout with the same values, against the oracle's GEMV, at a GEMV-sized and a tile-sized m."""
    from strands_decider.engine import QWeight
    n, k = 1152, 2048
    rng = np.random.default_rng(bits * 1000 + group + m + 7 * asym)
    packed, scales = M._quant_tensor(rng, n, k, bits, 1.0 / np.sqrt(k), group=group)
    bias = M._asym_bias(rng, scales, bits) if asym else None
    a = rng.standard_normal((m, k)).astype(np.float16)
    want = oracle.matmul(a, packed, scales, n, k, bits, group=group, variant=1, b=bias).astype(np.float32)
    q_d, s_d, a_d = dev(torch, packed), dev(torch, scales.view(np.uint16)), dev(torch, a.view(np.uint16))
    b_d = dev(torch, bias.view(np.uint16)) if asym else None
    w = QWeight(q_d.data_ptr(), s_d.data_ptr(), n, k, bits=bits, group=group, b_dev=b_d.data_ptr() if asym else None)
    y = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    w.matmul(a_d.data_ptr(), m, y.data_ptr(), n)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float32)
    err = np.abs(got - want)
    assert err.max() <= 2e-3 + 2e-3 * np.abs(want).max(), err.max()


@pytest.mark.parametrize("m,n,k,silu", [(2500, 2048, 2048, False), (1000, 8256, 2048, False), (777, 12288, 2048, True),
                                         (4097, 384, 192, False)])
def test_matmul_large_m(torch, m, n, k, silu):
    """Large token counts without split-K: many waves of persistent tiles, an odd count of 128-row
    weight tiles, an odd k-tile count, and the SwiGLU epilogue."""
    from strands_decider.engine import QWeight
    rng = np.random.default_rng(m + n + k)
    packed, scales = M._quant_tensor(rng, n, k, 4, 1.0 / np.sqrt(k))
    a = rng.standard_normal((m, k)).astype(np.float16)
    want = oracle.matmul(a, packed, scales, n, k, 4, variant=2).astype(np.float32)
    if silu:
        g, u = want[:, :n // 2], want[:, n // 2:]
        want = (g / (1 + np.exp(-g)) * u).astype(np.float16).astype(np.float32)
    q_d, s_d, a_d = dev(torch, packed), dev(torch, scales.view(np.uint16)), dev(torch, a.view(np.uint16))
    w = QWeight(q_d.data_ptr(), s_d.data_ptr(), n, k, interleave=silu)
    nout = n // 2 if silu else n
    y = torch.full((m, nout), float("nan"), dtype=torch.float16, device="cuda")
    w.matmul(a_d.data_ptr(), m, y.data_ptr(), nout, silu=silu, ws_dev=None, ws_bytes=0)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float32)
    assert np.isfinite(got).all()
    tol = (4e-3 if silu else 2e-3) * (1 + np.abs(want).max())
    assert np.abs(got - want).max() <= tol


@pytest.mark.parametrize("m", [5, 64, 100, 200, 328])
def test_matmul_swiglu_epilogue(torch, m):
    from strands_decider.engine import QWeight
    rng = np.random.default_rng(m)
    n, k = 2 * 6144, 2048
    packed, scales = M._quant_tensor(rng, n, k, 4, 1.0 / np.sqrt(k))
    a = rng.standard_normal((m, k)).astype(np.float16)
    big = oracle.matmul(a, packed, scales, n, k, 4, variant=2).astype(np.float32)
    g, u = big[:, :n // 2], big[:, n // 2:]
    want = (g / (1 + np.exp(-g)) * u).astype(np.float16).astype(np.float32)
    q_d, s_d, a_d = dev(torch, packed), dev(torch, scales.view(np.uint16)), dev(torch, a.view(np.uint16))
    w = QWeight(q_d.data_ptr(), s_d.data_ptr(), n, k, interleave=True)
    y = torch.zeros((m, n // 2), dtype=torch.float16, device="cuda")
    ws = torch.zeros(16 << 20, dtype=torch.float32, device="cuda")
    for ws_bytes in (0, ws.numel() * 4):
        w.matmul(a_d.data_ptr(), m, y.data_ptr(), n // 2, silu=True, ws_dev=ws.data_ptr(), ws_bytes=ws_bytes)
        torch.cuda.synchronize()
        got = y.cpu().numpy().astype(np.float32)
        assert np.abs(got - want).max() <= 4e-3 + 4e-3 * np.abs(want).max()


@pytest.mark.parametrize("l,p", [(300, 0), (37, 500), (1, 100), (129, 0), (60, 2048)])
@pytest.mark.parametrize("splits", [None, 0, 3, 7])  # None: sd_attention; else sd_attention_split (0: auto)
def test_attention_matches_oracle(torch, l, p, splits):
    from strands_decider.engine import attention
    rng = np.random.default_rng(l + p)
    hq, hk, hd, lt = 8, 2, 256, 4096
    q = rng.standard_normal((hq, l, hd)).astype(np.float16)
    kc = np.zeros((hk, lt, hd), np.float16)
    vc = np.zeros((hk, lt, hd), np.float16)
    kc[:, :p + l] = rng.standard_normal((hk, p + l, hd))
    vc[:, :p + l] = rng.standard_normal((hk, p + l, hd))
    kc[:, p + l:] = np.nan  # rows past the valid keys must never be read
    vc[:, p + l:] = np.nan
    gate = rng.standard_normal((l, 5120)).astype(np.float16)
    want = oracle.attn(q, kc[:, :p + l], vc[:, :p + l], gate, 5120, hd, 2 * hd, p=p).astype(np.float32)
    out = torch.zeros((l, hq * hd), dtype=torch.float16, device="cuda")
    qd, kd, vd, gd = (dev(torch, x.view(np.uint16)) for x in (q, kc, vc, gate))
    ws = torch.empty(32 << 20, dtype=torch.uint8, device="cuda")
    attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), gd.data_ptr(), 5120, hd, 2 * hd, out.data_ptr(), l, p, lt, hq, hk, hd,
              splits=splits, ws=ws.data_ptr(), ws_bytes=ws.numel())
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() < 4e-3


@pytest.mark.parametrize("l,p,hq,hk,gated", [(128, 0, 8, 2, True), (2048, 0, 8, 2, True), (200, 700, 8, 2, True),
                                             (1000, 3000, 8, 2, True), (513, 17, 16, 2, False), (130, 1, 4, 4, True)])
def test_attention_tc_matches_oracle(torch, l, p, hq, hk, gated):
    """sd_attention on query blocks of 128 (the tcgen05 kernel: l >= 128) against the oracle and against
    the mma.sync kernel (sd_attention_split with one split) on the same inputs: prefills, continuations
    of long prefixes, ragged last blocks, other head ratios, no gate."""
    from strands_decider.engine import attention
    rng = np.random.default_rng(l * 3 + p)
    hd, lt = 256, 4096
    q = rng.standard_normal((hq, l, hd)).astype(np.float16)
    kc = np.full((hk, lt, hd), np.nan, np.float16)  # rows past the valid keys must never be read
    vc = np.full((hk, lt, hd), np.nan, np.float16)
    kc[:, :p + l] = rng.standard_normal((hk, p + l, hd))
    vc[:, :p + l] = rng.standard_normal((hk, p + l, hd))
    gw = 3 * hq * hd
    gate = rng.standard_normal((l, gw)).astype(np.float16)
    if gated:
        want = oracle.attn(q, kc[:, :p + l], vc[:, :p + l], gate, gw, hd, 2 * hd, p=p).astype(np.float32)
    else:
        want = oracle.attn(q, kc[:, :p + l], vc[:, :p + l], None, 0, 0, 0, p=p).astype(np.float32)
    qd, kd, vd, gd = (dev(torch, x.view(np.uint16)) for x in (q, kc, vc, gate))
    ws = torch.empty(32 << 20, dtype=torch.uint8, device="cuda")
    outs = []
    for splits in (None, 1):
        out = torch.zeros((l, hq * hd), dtype=torch.float16, device="cuda")
        attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), gd.data_ptr() if gated else None, gw, hd, 2 * hd, out.data_ptr(),
                  l, p, lt, hq, hk, hd, splits=splits, ws=ws.data_ptr(), ws_bytes=ws.numel())
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy().astype(np.float32))
    tc, legacy = outs
    assert np.isfinite(tc).all()
    assert np.abs(tc - want).max() < 4e-3
    assert np.abs(tc - legacy).max() < 4e-3


@pytest.mark.parametrize("l,p", [(256, 0), (300, 44), (60, 10)])
def test_attention_batch_matches_one_by_one(torch, l, p):
    """sd_attention_batch (one launch over the batch) equals sd_attention on each sequence."""
    from strands_decider.engine import attention, attention_batch
    rng = np.random.default_rng(l + 7 * p)
    B, hq, hk, hd, lt = 3, 8, 2, 256, 512
    q = rng.standard_normal((B, hq, l, hd)).astype(np.float16)
    kc = rng.standard_normal((B, hk, lt, hd)).astype(np.float16)
    vc = rng.standard_normal((B, hk, lt, hd)).astype(np.float16)
    gate = rng.standard_normal((B, l, 3 * hq * hd)).astype(np.float16)
    qd, kd, vd, gd = (dev(torch, x.view(np.uint16)) for x in (q, kc, vc, gate))
    out = torch.zeros((B, l, hq * hd), dtype=torch.float16, device="cuda")
    attention_batch(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), gd.data_ptr(), 3 * hq * hd, hd, 2 * hd, out.data_ptr(), B, l, p,
                    lt, hq, hk, hd)
    one = torch.zeros((l, hq * hd), dtype=torch.float16, device="cuda")
    for b in range(B):
        attention(qd[b].data_ptr(), kd[b].data_ptr(), vd[b].data_ptr(), gd[b].data_ptr(), 3 * hq * hd, hd, 2 * hd, one.data_ptr(),
                  l, p, lt, hq, hk, hd)
        torch.cuda.synchronize()
        assert torch.equal(out[b], one)


def _gdn_inputs(rng, b, l, h):
    q = rng.standard_normal((b, l, h, 128)).astype(np.float32)
    k = rng.standard_normal((b, l, h, 128)).astype(np.float32)
    v = rng.standard_normal((b, l, h, 128)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, l, h))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((b, l, h))))).astype(np.float32)  # -softplus(N(0,1))
    s0 = (0.3 * rng.standard_normal((b, h, 128, 128))).astype(np.float32)
    return q, k, v, beta, g, s0


def test_gdn_serial_matches_oracle(torch):
    """The token-serial kernel against the oracle's recurrence (both f32, same order of operations
    up to the reductions): 1e-4."""
    from strands_decider.engine import gdn
    q, k, v, beta, g, s0 = _gdn_inputs(np.random.default_rng(11), 1, 200, 16)
    decay = np.exp(g)
    for load in (False, True):
        o_want, s_want = oracle.gdn(q[0], k[0], v[0], beta[0], decay[0], s0[0] if load else None)
        qd, kd, vd, bd, gd = (dev(torch, x) for x in (q, k, v, beta, g))
        sd_ = dev(torch, s0.copy())
        od = torch.zeros((200, 16 * 128), dtype=torch.float32, device="cuda")
        gdn(qd.data_ptr(), kd.data_ptr(), 2048, vd.data_ptr(), 2048, bd.data_ptr(), gd.data_ptr(), sd_.data_ptr(), load,
            od.data_ptr(), 200, 16, serial=True)
        torch.cuda.synchronize()
        np.testing.assert_allclose(od.cpu().numpy(), o_want, rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(sd_.cpu().numpy()[0], s_want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("b,l,in_f16,load", [(1, 200, False, False), (1, 64, False, True), (1, 7, False, True),
                                              (3, 130, True, True), (9, 333, True, False)])
def test_gdn_chunked_matches_oracle(torch, b, l, in_f16, load):
    """The chunked scan (tensor-core products on f16 operands, f32 accumulation and state) against the
    oracle's f32 recurrence: relative error of outputs and final state below 5e-3."""
    from strands_decider.engine import gdn
    h = 16
    q, k, v, beta, g, s0 = _gdn_inputs(np.random.default_rng(l + b), b, l, h)
    if in_f16:
        q, k, v = (x.astype(np.float16) for x in (q, k, v))
    qd, kd, vd, bd, gd = (dev(torch, x) for x in (q, k, v, beta, g))
    sd_ = dev(torch, s0.copy())
    od = torch.zeros((b, l, h * 128), dtype=torch.float32, device="cuda")
    gdn(qd.data_ptr(), kd.data_ptr(), h * 128, vd.data_ptr(), h * 128, bd.data_ptr(), gd.data_ptr(), sd_.data_ptr(), load,
        od.data_ptr(), l, h, batch=b, seq_qk=l * h * 128, seq_v=l * h * 128, in_f16=in_f16)
    torch.cuda.synchronize()
    got_o, got_s = od.cpu().numpy(), sd_.cpu().numpy()
    for i in range(b):
        o_want, s_want = oracle.gdn(q[i].astype(np.float32), k[i].astype(np.float32), v[i].astype(np.float32), beta[i],
                                    np.exp(g[i]), s0[i] if load else None)
        eo = np.linalg.norm(got_o[i] - o_want) / np.linalg.norm(o_want)
        es = np.linalg.norm(got_s[i] - s_want) / np.linalg.norm(s_want)
        assert eo < 5e-3 and es < 5e-3, (i, eo, es)
        assert np.abs(got_o[i] - o_want).max() < 3e-2


@pytest.mark.parametrize("b,l,load,algo", [(1, 1, True, 0), (2, 7, True, 0), (1, 63, False, 0), (3, 64, True, 0),
                                            (2, 65, False, 0), (4, 129, True, 0), (1, 1000, True, 0), (2, 130, True, 3)])
def test_gdn_f16_scans_match_oracle(torch, b, l, load, algo):
    """The f16 single-pass scans: algo 0 (the fused tcgen05 kernel: one CTA per sequence and head, all
    value columns) and 3 (mma.sync), over ragged last chunks, a single token, exact chunk multiples,
    batches with and without an entry state, against the oracle's recurrence: relative error below
    5e-3, and the batch's other sequences untouched by each one's padding rows."""
    from strands_decider.engine import gdn
    h = 16
    q, k, v, beta, g, s0 = _gdn_inputs(np.random.default_rng(7 * l + b + algo), b, l, h)
    q, k, v = (x.astype(np.float16) for x in (q, k, v))
    qd, kd, vd, bd, gd = (dev(torch, x) for x in (q, k, v, beta, g))
    sd_ = dev(torch, s0.copy())
    od = torch.full((b, l, h * 128), float("nan"), dtype=torch.float32, device="cuda")
    gdn(qd.data_ptr(), kd.data_ptr(), h * 128, vd.data_ptr(), h * 128, bd.data_ptr(), gd.data_ptr(), sd_.data_ptr(), load,
        od.data_ptr(), l, h, batch=b, seq_qk=l * h * 128, seq_v=l * h * 128, in_f16=True, algo=algo)
    torch.cuda.synchronize()
    got_o, got_s = od.cpu().numpy(), sd_.cpu().numpy()
    assert np.isfinite(got_o).all() and np.isfinite(got_s).all()
    for i in range(b):
        o_want, s_want = oracle.gdn(q[i].astype(np.float32), k[i].astype(np.float32), v[i].astype(np.float32), beta[i],
                                    np.exp(g[i]), s0[i] if load else None)
        eo = np.linalg.norm(got_o[i] - o_want) / np.linalg.norm(o_want)
        es = np.linalg.norm(got_s[i] - s_want) / np.linalg.norm(s_want)
        assert eo < 5e-3 and es < 5e-3, (i, eo, es)


@pytest.mark.parametrize("l,load", [(333, False), (64, True), (65, True), (1000, True)])
def test_gdn_two_phase_matches_oracle(torch, l, load):
    """The two-phase scan (all chunks' intra-chunk products in parallel, then the state walk) against
    the oracle's recurrence, one sequence with f16 inputs: relative error below 5e-3."""
    from strands_decider.engine import GDN_TWO_PHASE, gdn, gdn_scratch_bytes
    h = 16
    q, k, v, beta, g, s0 = _gdn_inputs(np.random.default_rng(l * 3 + load), 1, l, h)
    q, k, v = (x.astype(np.float16) for x in (q, k, v))
    qd, kd, vd, bd, gd = (dev(torch, x) for x in (q, k, v, beta, g))
    sd_ = dev(torch, s0.copy())
    od = torch.zeros((l, h * 128), dtype=torch.float32, device="cuda")
    nb = gdn_scratch_bytes(l, h)
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    gdn(qd.data_ptr(), kd.data_ptr(), h * 128, vd.data_ptr(), h * 128, bd.data_ptr(), gd.data_ptr(), sd_.data_ptr(), load,
        od.data_ptr(), l, h, in_f16=True, algo=GDN_TWO_PHASE, scratch=scratch.data_ptr(), scratch_bytes=nb)
    torch.cuda.synchronize()
    o_want, s_want = oracle.gdn(q[0].astype(np.float32), k[0].astype(np.float32), v[0].astype(np.float32), beta[0],
                                np.exp(g[0]), s0[0] if load else None)
    got_o, got_s = od.cpu().numpy(), sd_.cpu().numpy()[0]
    eo = np.linalg.norm(got_o - o_want) / np.linalg.norm(o_want)
    es = np.linalg.norm(got_s - s_want) / np.linalg.norm(s_want)
    assert eo < 5e-3 and es < 5e-3, (eo, es)


@pytest.fixture(scope="module")
def engines(small_model):
    from strands_decider.engine import Engine
    return Engine.load(small_model), oracle.Engine(small_model)


@pytest.mark.parametrize("l", [9, 40, 300])
def test_engine_layers_match_oracle(engines, l):
    gpu, cpu = engines
    rng = np.random.default_rng(l)
    ids = rng.integers(0, 8192, l)
    rows = sorted(set([0, l // 2, l - 1]))
    out = gpu.forward(ids, rows, trace=True)
    want, _, tr = cpu.forward(ids, rows, trace=True)
    per_layer = np.abs(out.trace - tr).max(axis=(1, 2))
    assert per_layer.max() < 2e-2, per_layer
    assert np.abs(out.hidden - want).max() < 2e-2


def test_engine_probabilities_match_oracle(engines, small_model):
    from strands_decider.engine import Head
    gpu, cpu = engines
    head = Head.load(f"{small_model}/head.safetensors")
    tensors = M.read_safetensors(f"{small_model}/head.safetensors")
    rng = np.random.default_rng(3)
    worst = 0.0
    for case in range(12):
        l = int(rng.integers(20, 400))
        ids = rng.integers(0, 8192, l)
        nopt = int(rng.integers(2, 6))
        rows = sorted(rng.choice(l - 1, nopt, replace=False).tolist()) + [l - 1]
        a = head.probs(gpu.forward(ids, rows).hidden, 2048, 1.0)
        b = oracle.head_probs(cpu.forward(ids, rows)[0], tensors, 1.0)
        worst = max(worst, np.abs(a - b).max())
        assert np.argmax(a) == np.argmax(b)
    assert worst < 1e-3, worst


def test_prefix_cache_matches_full_forwards(engines):
    """`tests/engine_parity.rs:59-85` on the GPU engine: max |dp| < 2e-3."""
    from strands_decider.engine import Head
    gpu, _ = engines
    rng = np.random.default_rng(5)
    state = rng.integers(0, 8000, 150)
    snap = gpu.forward(state, [], keep=True).snapshot
    assert snap.len == 150
    for ql in (24, 48, 7):
        q = rng.integers(0, 8000, ql)
        rows = [2, ql // 2, ql - 1]
        a = gpu.forward(q, rows, cache=snap).hidden
        b = gpu.forward(np.concatenate([state, q]), [150 + r for r in rows]).hidden
        assert np.abs(a - b).max() < 2e-2
    # the snapshot is immutable: the same continuation twice is bit-identical
    q = rng.integers(0, 8000, 30)
    a = gpu.forward(q, [29], cache=snap).hidden
    b = gpu.forward(q, [29], cache=snap).hidden
    assert np.array_equal(a, b)
    snap.close()


def test_snapshot_of_continuation(engines):
    gpu, cpu = engines
    rng = np.random.default_rng(9)
    s1, s2, q = rng.integers(0, 8000, 60), rng.integers(0, 8000, 40), rng.integers(0, 8000, 25)
    a = gpu.forward(s1, [], keep=True).snapshot
    b = gpu.forward(s2, [], cache=a, keep=True).snapshot
    assert b.len == 100
    got = gpu.forward(q, [24], cache=b).hidden
    want = cpu.forward(np.concatenate([s1, s2, q]), [124])[0]
    assert np.abs(got - want).max() < 2e-2


def test_full_context_forward(engines):
    """The maximum context (4096 tokens, `src/engine.rs:532`): one forward of all of it, the same
    tokens as a 4000-token snapshot plus a 96-token continuation ending exactly at the limit (the
    reference's prefix forward == full forward invariant, `tests/engine_parity.rs:59-85`), and the
    same sequence packed beside a short one in one batch."""
    gpu, _ = engines
    rng = np.random.default_rng(4096)
    ids = rng.integers(0, 8000, 4096)
    rows = [0, 2047, 4000, 4095]
    full = gpu.forward(ids, rows).hidden
    assert np.isfinite(full).all()
    snap = gpu.forward(ids[:4000], [], keep=True).snapshot
    cont = gpu.forward(ids[4000:], [0, 95], cache=snap).hidden
    assert np.abs(cont - full[2:]).max() < 2e-2
    snap.close()
    outs, _ = gpu.forward_batch(None, [rng.integers(0, 8000, 37), ids], [[36], rows])
    assert np.abs(outs[1] - full).max() < 2e-2


def test_engine_errors(engines):
    from strands_decider.engine import Error
    gpu, _ = engines
    with pytest.raises(Error, match="out of range"):
        gpu.forward([1, 2, 3], [3])
    with pytest.raises(Error, match="context of"):
        gpu.forward(np.zeros(4097, np.int64), [])
    with pytest.raises(Error, match="token id"):
        gpu.forward([1, 999999], [0])
    snap = gpu.forward(np.zeros(4000, np.int64), [], keep=True).snapshot
    with pytest.raises(Error, match="context of"):
        gpu.forward(np.zeros(100, np.int64), [0], cache=snap)
    # the engine still works after the failures
    assert gpu.forward([5, 6, 7], [2]).hidden.shape == (1, 2048)


def test_decider_answers_match_oracle(small_model):
    """`Decider::ask_all` through the GPU engine against the same pipeline through the oracle."""
    from strands_decider import Decider, Question
    from strands_decider import prompt
    dec = Decider.load(small_model)
    state = "Help! My payouts have been failing for 3 days! " * 3
    qs = [Question.noul("Does this convey urgency?"),
          Question.choice("Which team should handle this?", ["billing", "technical", "sales"]),
          Question.score("How frustrated is the writer?", ["calm", "frustrated", "very angry"])]
    answers = dec.ask_all(state, qs)
    named = [(str(i), q) for i, q in enumerate(qs)]
    rendered, sids, qencs, options = dec.encode(state, named)
    cpu = oracle.Engine(small_model)
    tensors = M.read_safetensors(f"{small_model}/head.safetensors")
    snap = cpu.forward(sids, [], keep=True)[1]
    for i, (q, a) in enumerate(zip(qencs, answers)):
        rows = list(options[i]) + [len(q.ids) - 1]
        probs = oracle.head_probs(cpu.forward(q.ids, rows, cache=snap)[0], tensors, 1.0)
        want = prompt.to_answer(rendered[i], probs, 0.0)
        got_p = dict(a.probabilities) if a.probabilities else {"true": a.noul}
        want_p = dict(want.probabilities) if want.probabilities else {"true": want.noul}
        for kk in want_p:
            assert abs(got_p[kk] - want_p[kk]) <= 1e-3 + 1e-4  # 4-decimal rounding on both sides
        if a.kind == "choice":
            assert a.choice == want.choice
    one = dec.ask(state, qs[1])
    assert one.kind == "choice"
