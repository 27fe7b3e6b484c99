"""Two-sided Gaussian sketches of large matrices for the golden fixtures: S = W_l^T X W_r (16 x 16), W_l and W_r
standard normal, seeded by the matrix's dimensions alone. For any X, E||W_l^T X W_r||_F^2 = 256 ||X||_F^2, so the
relative error between the sketches of two matrices estimates their relative Frobenius error (the difference
sketched like any matrix) while a fixture stores 256 numbers instead of the whole matrix. Vectors (1-D) are kept
whole. Used by tests/golden/make_golden.py (sketching the reference's outputs) and by the parity tests (sketching
the B200 outputs the same way)."""
import numpy as np

K_SKETCH = 16


def omega(n, side):
    return np.random.default_rng([int(n), 7 if side == "l" else 11]).standard_normal((int(n), K_SKETCH))


def sketch(X):
    X = np.asarray(X, dtype=np.float64)
    if X.ndim < 2:
        return X.reshape(-1).copy()
    X = X.reshape(X.shape[0], -1)
    return omega(X.shape[0], "l").T @ X @ omega(X.shape[1], "r")
