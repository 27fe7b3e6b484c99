"""Host encoding of the layout changes of order-r parameters (psgd_pro_b200.optimizer._permute_item): the output
index -> source index walk that the permute kernel does, replayed here in numpy over the encoded fields, must move
a tensor exactly as numpy's moveaxis does, with the diagonal scales multiplied in (no GPU: the CUDA kernel itself
is checked by the N-D step parity on the device)."""
import itertools

import numpy as np
import pytest
import torch

from psgd_pro_b200 import _capi
from psgd_pro_b200.optimizer import _permute_item


def replay(it, src_flat):
    """What permute_kernel computes for every output index f (nd_kernels.cu pm_value)."""
    out = np.empty(it.numel)
    for f in range(it.numel):
        rest, s, v = f, 0, 1.0
        for p in range(it.order - 1, -1, -1):
            d = it.odim[p]
            i = rest % d
            rest //= d
            m = it.omode[p]
            s += i * it.sstride[m]
            if it.scale[m]:
                v *= SCALES[m][i]
        out[f] = src_flat[s] * v
    return out


SCALES = {}


def layout(x, mode, first=False):
    """x (natural dims) in the layout with `mode` moved to the end (or front), flattened."""
    if mode is None:
        return x.reshape(-1)
    return np.moveaxis(x, mode, 0 if first else -1).reshape(-1)


@pytest.mark.parametrize("dims", [(3, 4, 5), (2, 3, 2, 4), (5, 1, 3)])
def test_permute_encoding_moves_modes_like_numpy(dims):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(dims)
    r = len(dims)
    src_t = torch.zeros(x.size)  # only its data pointer is encoded
    for src_last, dst in itertools.product([None] + list(range(r)), [None] + list(range(r))):
        for first in ([False, True] if dst is not None else [False]):
            SCALES.clear()
            scales = [None] * r
            want = x.copy()
            if src_last is None and r > 1:  # one diagonal scale, on mode 1
                sc = torch.arange(1, dims[1] + 1, dtype=torch.float32)
                scales[1] = sc
                SCALES[1] = sc.numpy()
                shp = [1] * r
                shp[1] = -1
                want = want * SCALES[1].reshape(shp)
            it, units = _permute_item(src_t, dims, src_last, dst, first, scales)
            got = replay(it, layout(x, src_last))
            np.testing.assert_allclose(got, layout(want, dst, first), rtol=1e-6)
            if dst is not None and not first:
                assert it.cols == dims[dst]
            if dst is not None and first:
                assert it.cols == x.size // dims[dst]
            assert units == -(-x.size // _capi.PERMUTE_CHUNK)
