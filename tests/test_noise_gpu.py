"""In-kernel damping noise of psgd_prep (hyper[PSGD_HY_NOISE] set) against the test-side restatement of its
generator (tests/noise_ref.py): with G = 0, damping 1 and eps 0 the staged operand is the noise itself."""
import ctypes
import struct

import numpy as np
import pytest
import torch

from noise_ref import normals
from psgd_pro_b200 import _capi
from psgd_pro_b200 import kernels as K

pytestmark = pytest.mark.gpu


def staged_noise(dev, n1, n2, mode, base, key, split=True, g_dtype=torch.float32):
    g = torch.zeros(n1, n2, device=dev, dtype=g_dtype)
    dummy = torch.zeros(4, device=dev)  # any non-null xi marks the item as one with damping noise
    rows, cols = (n2, n1) if mode == _capi.PSGD_PREP_TRANS else (n1, n2)
    hi, lo = K.operand(rows, cols, dev, split=split)
    it = _capi.PrepItem()
    it.g, it.g_bf16 = g.data_ptr(), int(g_dtype == torch.bfloat16)
    it.mode, it.xi, it.n1, it.n2 = mode, dummy.data_ptr(), n1, n2
    it.out_hi, it.out_lo, it.ld_out, it.eps, it.noise_base = K.ptr(hi), K.ptr(lo), hi.stride(0), 0.0, base
    host = torch.empty(ctypes.sizeof(it), dtype=torch.uint8)
    ctypes.memmove(host.data_ptr(), ctypes.addressof(it), ctypes.sizeof(it))
    items = host.to(dev)
    if mode == _capi.PSGD_PREP_NORMAL:
        pairs = [(0, rb) for rb in range((n1 + _capi.PREP_ROWS - 1) // _capi.PREP_ROWS)]
    else:
        pairs = [(0, (ti << 16) | tj) for ti in range((n1 + 31) // 32) for tj in range((n2 + 31) // 32)]
    work = torch.tensor([v for p in pairs for v in p], dtype=torch.int32).to(dev)
    bits = [0] * _capi.HY_COUNT
    bits[_capi.HY_DAMPING] = struct.unpack("<i", struct.pack("<f", 1.0))[0]
    bits[_capi.HY_NOISE] = struct.unpack("<i", struct.pack("<f", 1.0))[0]
    bits[_capi.HY_NOISE_KEY0], bits[_capi.HY_NOISE_KEY1] = (struct.unpack("<i", struct.pack("<I", k))[0] for k in key)
    hyper = torch.tensor(bits, dtype=torch.int32).to(dev).view(torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _capi.check(_capi.lib().psgd_prep(items.data_ptr(), work.data_ptr(), len(pairs), hyper.data_ptr(), err.data_ptr(),
                                      K.stream_handle()), "psgd_prep")
    torch.cuda.synchronize()
    assert err.item() == 0
    z = hi[:, :cols].float() + (lo[:, :cols].float() if lo is not None else 0)
    return z.cpu().double().numpy()


@pytest.mark.parametrize("n1,n2,base", [(96, 1000, 0), (40, 37, 12), (300, 64, 4 * 12345)])
def test_noise_matches_reference(cuda, n1, n2, base):
    key = (0x1234567, 42)
    z = staged_noise(cuda, n1, n2, _capi.PSGD_PREP_NORMAL, base, key)
    want = normals(base + np.arange(n1 * n2), *key).reshape(n1, n2)
    assert np.abs(z - want).max() < 2e-4 * max(1.0, np.abs(want).max())
    zt = staged_noise(cuda, n1, n2, _capi.PSGD_PREP_TRANS, base, key)  # another launch geometry: same numbers
    assert np.abs(zt.T - z).max() < 1e-6 * max(1.0, np.abs(z).max())
    zb = staged_noise(cuda, n1, n2, _capi.PSGD_PREP_NORMAL, base, key, g_dtype=torch.bfloat16)  # bf16 G path
    assert np.array_equal(zb, z)


def test_noise_keys_and_moments(cuda):
    a = staged_noise(cuda, 512, 512, _capi.PSGD_PREP_NORMAL, 0, (7, 1))
    b = staged_noise(cuda, 512, 512, _capi.PSGD_PREP_NORMAL, 0, (7, 1))
    c = staged_noise(cuda, 512, 512, _capi.PSGD_PREP_NORMAL, 0, (7, 2))
    assert np.array_equal(a, b)
    assert abs(np.corrcoef(a.ravel(), c.ravel())[0, 1]) < 0.01
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1) < 0.01
