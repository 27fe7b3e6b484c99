"""psgd_trace (sum of S o Q for the Procrustes step size) through the C ABI against an fp64 torch sum of the same
stored S (bf16 hi, plus lo when given) and fp32 Q: vector rows, n % 8 == 4 tails, odd n (element path), several
items in one launch."""
import ctypes

import pytest
import torch

from psgd_pro_b200 import _capi
from psgd_pro_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _upload(items, dev):
    arr = (_capi.TraceItem * len(items))(*items)
    host = torch.empty(ctypes.sizeof(arr), dtype=torch.uint8)
    ctypes.memmove(host.data_ptr(), ctypes.addressof(arr), ctypes.sizeof(arr))
    return host.to(dev)


@pytest.mark.parametrize("split", [False, True])
def test_trace_matches_fp64(cuda, split):
    g = torch.Generator().manual_seed(3)
    sizes = [96, 100, 37, 300, 8, 1]
    items, work, keep, want = [], [], [], []
    for k, n in enumerate(sizes):
        q = torch.randn(n, n, generator=g).to(cuda)
        S = torch.randn(n, n, generator=g).to(cuda)
        hi, lo = K.operand(n, n, cuda, split=split)
        K.split_into(S, hi, lo) if split else hi[:, :n].copy_(S.to(torch.bfloat16))
        it = _capi.TraceItem()
        part = torch.full((-(-n // _capi.TRACE_ROWS),), float("nan"), device=cuda)
        it.q, it.n, it.s_hi, it.s_lo, it.lds, it.part = q.data_ptr(), n, K.ptr(hi), K.ptr(lo), hi.stride(0), part.data_ptr()
        items.append(it)
        work += [(k, r0) for r0 in range(0, n, _capi.TRACE_ROWS)]
        stored = hi[:, :n].double() + (lo[:, :n].double() if split else 0)
        want.append((stored * q.double()).sum().item())
        keep += [q, S, hi, lo, part]
    dev_items = _upload(items, cuda)
    w = torch.tensor([v for p in work for v in p], dtype=torch.int32).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(2):  # a second launch over the same buffers gives the same sums
        _capi.check(_capi.lib().psgd_trace(dev_items.data_ptr(), w.data_ptr(), len(work), int(split),
                                           err.data_ptr(), K.stream_handle()), "psgd_trace")
        torch.cuda.synchronize()
        assert err.item() == 0
        for k, n in enumerate(sizes):
            part = keep[5 * k + 4]
            got = part.double().sum().item()
            scale = (keep[5 * k + 2][:, :n].double().abs() * keep[5 * k].double().abs()).sum().item()
            assert abs(got - want[k]) <= 1e-6 * scale, (n, got, want[k])
