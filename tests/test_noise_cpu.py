"""The test-side Philox4x32-10 (tests/noise_ref.py) reproduces the generator's published known-answer vectors."""
import numpy as np

from noise_ref import normals, philox4x32_10


def test_philox_known_answers():
    kat = [([0, 0, 0, 0], [0, 0], [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
           ([0xffffffff] * 4, [0xffffffff] * 2, [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
           ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0],
            [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1])]
    for c, k, want in kat:
        assert philox4x32_10(c, k).tolist() == want


def test_normals_look_standard():
    z = normals(np.arange(200_000), 12345, 7)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    assert abs(np.corrcoef(z[:-1], z[1:])[0, 1]) < 0.01
