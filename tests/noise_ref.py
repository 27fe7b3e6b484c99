"""Test-side restatement of the in-kernel damping-noise generator (psgd_prep with hyper[PSGD_HY_NOISE] set):
Philox4x32-10 (Salmon, Moraes, Dror and Shaw, SC'11) on counter (s / 4, 0, 0, 0) with a 2-word key, the four words
turned into uniforms ((w >> 9) + 1/2) / 2^23 and four standard normal numbers by two Box-Muller transforms (angles
2 pi u - pi). numpy, float64 transforms."""
import numpy as np

M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32_10(c, k):
    """c: (..., 4) uint64 counters (32-bit values), k: (k0, k1). Returns (..., 4) uint64 words."""
    c = np.array(c, dtype=np.uint64)
    k0, k1 = np.uint64(k[0]), np.uint64(k[1])
    m = np.uint64(MASK)
    for _ in range(10):
        p0 = np.uint64(M0) * c[..., 0]
        p1 = np.uint64(M1) * c[..., 2]
        c = np.stack([((p1 >> np.uint64(32)) & m) ^ c[..., 1] ^ k0, p1 & m,
                      ((p0 >> np.uint64(32)) & m) ^ c[..., 3] ^ k1, p0 & m], axis=-1)
        k0 = (k0 + np.uint64(W0)) & m
        k1 = (k1 + np.uint64(W1)) & m
    return c


def normals(positions, k0, k1):
    """Standard normal numbers at the given sequence positions (int64 array)."""
    pos = np.asarray(positions, dtype=np.uint64)
    blk = pos >> np.uint64(2)
    c = np.stack([blk & np.uint64(MASK), blk >> np.uint64(32), np.zeros_like(blk), np.zeros_like(blk)], axis=-1)
    w = philox4x32_10(c, (k0, k1))
    u = ((w >> np.uint64(9)).astype(np.float64) + 0.5) * 2.0 ** -23  # the top 23 bits of each word
    r0, r1 = np.sqrt(-2 * np.log(u[..., 0])), np.sqrt(-2 * np.log(u[..., 2]))
    t1, t3 = 2 * np.pi * u[..., 1] - np.pi, 2 * np.pi * u[..., 3] - np.pi
    z = np.stack([r0 * np.cos(t1), r0 * np.sin(t1), r1 * np.cos(t3), r1 * np.sin(t3)], axis=-1)
    return np.take_along_axis(z, (pos & np.uint64(3)).astype(np.int64)[..., None], axis=-1)[..., 0]
