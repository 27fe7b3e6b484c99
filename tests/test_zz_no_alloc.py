"""psgd_apply_noalloc, the clip + apply entry point for callers that cannot allocate device memory (a plugin whose
host owns all device allocations, code inside another framework's memory pool, a loop that cannot afford the
synchronisation of cudaMalloc), against psgd_apply, whose caller supplies the scratch.

Both run through the C ABI on the same inputs, twice in a row: the first call is large enough to clip, the second
is smaller, so the second reads fewer scratch slots than the first left behind. Results must agree within the
fp32 parity bar of the other GPU tests (1e-3 relative Frobenius; in practice they differ only in the order of the
sum of squares). This file is collected last, so a run that stops at the first failure has run every other test."""
import ctypes
import math

import pytest
import torch

from psgd_pro_b200 import _capi
from psgd_pro_b200._capi import APPLY_CHUNK, HY_COUNT, HY_LR_PARAMS, HY_MAX_AVG, HY_MAX_ELEM, ApplyItem
from psgd_pro_b200.kernels import stream_handle

pytestmark = pytest.mark.gpu

LR, MAX_AVG, MAX_ELEM = 0.01, 2.0, 10.0


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def apply_with_caller_scratch(param, pg):
    """The existing entry point: per-chunk sums of squares, the clip-scale slot and the item array are device
    memory allocated here by the caller."""
    numel = pg.numel()
    nch = math.ceil(numel / APPLY_CHUNK)
    padded = torch.zeros(nch * APPLY_CHUNK, device=pg.device)
    padded[:numel] = pg.reshape(-1)
    part = padded.view(nch, APPLY_CHUNK).pow(2).sum(1)
    scale = torch.zeros(1, device=pg.device)
    it = ApplyItem()
    it.param, it.param_bf16, it.numel = param.data_ptr(), int(param.dtype == torch.bfloat16), numel
    it.pg, it.part, it.nparts, it.scale = pg.data_ptr(), part.data_ptr(), nch, scale.data_ptr()
    host = torch.empty(ctypes.sizeof(it), dtype=torch.uint8)
    ctypes.memmove(host.data_ptr(), ctypes.addressof(it), ctypes.sizeof(it))
    items = host.to(pg.device)
    work = torch.tensor([v for c in range(nch) for v in (0, c)], dtype=torch.int32).to(pg.device)
    hyper = torch.zeros(HY_COUNT)
    hyper[HY_LR_PARAMS], hyper[HY_MAX_AVG], hyper[HY_MAX_ELEM] = LR, MAX_AVG, MAX_ELEM
    hyper = hyper.to(pg.device)
    err = torch.zeros(1, dtype=torch.int32, device=pg.device)
    rc = _capi.lib().psgd_apply(items.data_ptr(), 1, work.data_ptr(), nch, hyper.data_ptr(), err.data_ptr(),
                                stream_handle())
    _capi.check(rc, "psgd_apply")
    torch.cuda.synchronize()
    assert err.item() == 0


def reference_apply(p0, pg):
    """psgd_pro.py:371-381 restated in fp32 torch: scale Pg to RMS max_avg_amp when its RMS is larger, clamp each
    element to +-max_element_amp, param -= lr_params * Pg (a bf16 parameter is updated in fp32 and rounded back,
    as torch's subtract_ on a bf16 tensor does)."""
    g = pg.clone()
    avg = torch.sqrt(torch.mean(g * g))
    if avg > MAX_AVG:
        g *= MAX_AVG / avg
    g.clamp_(min=-MAX_ELEM, max=MAX_ELEM)
    return (p0.float() - LR * g).to(p0.dtype)


def apply_without_scratch(param, pg):
    rc = _capi.lib().psgd_apply_noalloc(param.data_ptr(), int(param.dtype == torch.bfloat16), pg.data_ptr(),
                                        pg.numel(), LR, MAX_AVG, MAX_ELEM, stream_handle())
    _capi.check(rc, "psgd_apply_noalloc")
    torch.cuda.synchronize()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_apply_on_two_calls_in_a_row(cuda, dtype):
    g = torch.Generator(device=cuda)
    g.manual_seed(7)
    # call 1: 3 M elements with RMS 3 (the average-amplitude clip fires); call 2: 70 k elements with RMS 0.5 and a
    # few large entries (no average clip, the element clamp fires)
    cases = [(3_000_001, 3.0), (70_000, 0.5)]
    for numel, rms in cases:
        pg = torch.randn(numel, device=cuda, generator=g) * rms
        if rms < 1:
            pg[::997] = 40.0
        p0 = (torch.randn(numel, device=cuda, generator=g) * 0.1).to(dtype)
        a, b = p0.clone(), p0.clone()
        apply_with_caller_scratch(a, pg)
        apply_without_scratch(b, pg)
        assert torch.isfinite(b.float()).all()
        assert rel(b.float() - p0.float(), a.float() - p0.float()) < 1e-3
        assert rel(b.float(), a.float()) < 1e-3
        # and directly against the reference's arithmetic (fp32 torch); a bf16 parameter may differ by one rounding
        # of the stored value where the two fp32 results straddle a bf16 rounding boundary
        r = reference_apply(p0, pg)
        bar = 1e-3 if dtype == torch.float32 else 2e-2
        assert rel(b.float() - p0.float(), r.float() - p0.float()) < bar
        assert rel(b.float(), r.float()) < 1e-3
        # the update really was clipped / clamped as the reference does (psgd_pro.py:371-381)
        step = (p0.float() - b.float()) / LR
        assert step.abs().max().item() <= MAX_ELEM * 1.01


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    lib = _capi.lib()
    x = torch.zeros(8, device=cuda)
    too_big = _capi.c_ll(4096 * APPLY_CHUNK + 1)
    rc = lib.psgd_apply_noalloc(x.data_ptr(), 0, x.data_ptr(), too_big, LR, MAX_AVG, MAX_ELEM, stream_handle())
    assert rc == -5
    assert lib.psgd_apply_noalloc(x.data_ptr(), 0, x.data_ptr(), 0, LR, MAX_AVG, MAX_ELEM, stream_handle()) == 0


def test_noalloc_propagates_nan_like_the_reference(cuda):
    """A NaN or an Inf in Pg reaches the parameter as NaN, as psgd_pro.py:371-381 does (Inf makes the RMS
    infinite, the scale 0 and Inf * 0 = NaN); a clipped update must not hide a diverging run."""
    pg = torch.randn(50_000, device=cuda) * 0.3
    pg[123] = float("nan")
    p0 = torch.randn(50_000, device=cuda) * 0.1
    for bad in (float("nan"), float("inf")):
        pg[123] = bad
        r = reference_apply(p0, pg)
        for fn in (apply_without_scratch, apply_with_caller_scratch):  # both entry points share the semantics
            b = p0.clone()
            fn(b, pg)
            assert torch.equal(torch.isnan(b), torch.isnan(r)) and bool(torch.isnan(b[123])), (fn.__name__, bad)
            fin = torch.isfinite(r)
            assert rel(b[fin], r[fin]) < 1e-6, (fn.__name__, bad)
