"""sd_gdn_noalloc: the gated-delta scan for callers that must not allocate device memory while they
run (for example a serving process whose GPU memory is all reserved when it starts, or a latency
path that cannot take cudaMalloc's implicit device synchronisation). Its scratch is one fixed array
inside the library shared by every call on a device, so the checks here are that two calls in a row
(the second reusing what the first left in the array) each give what the allocating entry point
gives, and that a call too large for the array is refused with a clear error.

This file is named to be collected last: it must pass on its own in a fresh process and after every
other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(rng, l, h):
    q = rng.standard_normal((l, h * 128)).astype(np.float16)
    k = rng.standard_normal((l, h * 128)).astype(np.float16)
    v = rng.standard_normal((l, h * 128)).astype(np.float16)
    beta = (1 / (1 + np.exp(-rng.standard_normal((l, h))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((l, h))))).astype(np.float32)
    s0 = (0.3 * rng.standard_normal((h, 128, 128))).astype(np.float32)
    return q, k, v, beta, g, s0


def test_noalloc_matches_the_allocating_scan_twice_in_a_row():
    import torch
    from strands_decider.engine import GDN_TWO_PHASE, gdn, gdn_noalloc, gdn_noalloc_max_tokens, gdn_scratch_bytes
    assert torch.cuda.is_available()
    h = 16
    lmax = gdn_noalloc_max_tokens(h)
    assert lmax == 1088
    rng = np.random.default_rng(21)
    # the first call fills 272 of the array's 278 chunk records (17 chunks x 16 heads); the second,
    # shorter one runs over what it left behind
    for l, load in ((lmax, True), (300, False)):
        q, k, v, beta, g, s0 = _inputs(rng, l, h)
        dq, dk, dv = (torch.from_numpy(x.view(np.uint16)).cuda() for x in (q, k, v))
        db, dg = torch.from_numpy(beta).cuda(), torch.from_numpy(g).cuda()
        outs = []
        for noalloc in (False, True):
            st = torch.from_numpy(s0.copy()).cuda()
            o = torch.zeros((l, h * 128), dtype=torch.float32, device="cuda")
            if noalloc:
                gdn_noalloc(dq.data_ptr(), dk.data_ptr(), h * 128, dv.data_ptr(), h * 128, db.data_ptr(), dg.data_ptr(),
                            st.data_ptr(), load, o.data_ptr(), l, h)
            else:
                nb = gdn_scratch_bytes(l, h)
                scr = torch.empty(nb, dtype=torch.uint8, device="cuda")
                gdn(dq.data_ptr(), dk.data_ptr(), h * 128, dv.data_ptr(), h * 128, db.data_ptr(), dg.data_ptr(),
                    st.data_ptr(), load, o.data_ptr(), l, h, in_f16=True, algo=GDN_TWO_PHASE, scratch=scr.data_ptr(),
                    scratch_bytes=nb)
            torch.cuda.synchronize()
            outs.append((o.cpu().numpy(), st.cpu().numpy()))
        (o_ref, s_ref), (o_na, s_na) = outs
        # the GDN tests' tolerance (relative error below 5e-3); the kernels are the same, so equal
        assert np.linalg.norm(o_na - o_ref) / np.linalg.norm(o_ref) < 5e-3
        assert np.linalg.norm(s_na - s_ref) / np.linalg.norm(s_ref) < 5e-3
        assert np.array_equal(o_na, o_ref) and np.array_equal(s_na, s_ref)


def test_noalloc_call_takes_no_device_memory():
    """Once a device has run a first call (which loads the library's gated-delta module and with it
    the fixed array), further calls leave the device's free memory exactly as it was."""
    import torch
    from strands_decider.engine import gdn_noalloc
    h, l = 16, 700
    rng = np.random.default_rng(5)
    q, k, v, beta, g, s0 = _inputs(rng, l, h)
    dq, dk, dv = (torch.from_numpy(x.view(np.uint16)).cuda() for x in (q, k, v))
    db, dg = torch.from_numpy(beta).cuda(), torch.from_numpy(g).cuda()
    st = torch.from_numpy(s0).cuda()
    o = torch.zeros((l, h * 128), dtype=torch.float32, device="cuda")
    args = (dq.data_ptr(), dk.data_ptr(), h * 128, dv.data_ptr(), h * 128, db.data_ptr(), dg.data_ptr(), st.data_ptr(), 1,
            o.data_ptr(), l, h)
    gdn_noalloc(*args)  # warm-up: the module (and the array) is resident after this
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    gdn_noalloc(*args)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert np.isfinite(o.cpu().numpy()).all()


def test_noalloc_refuses_sizes_beyond_its_scratch():
    import torch
    from strands_decider.engine import Error, gdn_noalloc, gdn_noalloc_max_tokens
    h = 16
    l = gdn_noalloc_max_tokens(h) + 1
    x = torch.zeros((l, h * 128), dtype=torch.float16, device="cuda")
    gates = torch.zeros((l, h), dtype=torch.float32, device="cuda")
    st = torch.zeros((h, 128, 128), dtype=torch.float32, device="cuda")
    o = torch.zeros((l, h * 128), dtype=torch.float32, device="cuda")
    with pytest.raises(Error, match="fixed scratch holds"):
        gdn_noalloc(x.data_ptr(), x.data_ptr(), h * 128, x.data_ptr(), h * 128, gates.data_ptr(), gates.data_ptr(),
                    st.data_ptr(), 0, o.data_ptr(), l, h)
