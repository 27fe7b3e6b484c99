"""CPU oracle of the PSGD-Kron (Q0.5EQ1.5 whitening) optimizer step: a numpy restatement of the reference's math.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg
may import this module, and only as the checker or the timed CPU baseline; the product path (psgd_pro_b200) never
does. Parity is pinned: tests/test_oracle_golden.py checks this module against golden vectors made by running the
reference itself (tests/golden/make_golden.py, with identical random draws).

Every function cites the reference lines it restates (paths relative to the reference repository). Random draws
are arguments, never drawn here, in the reference's order (psgd_pro_fast.py:200-206 draw_normals):
    per parameter: xi (shape of G), then for each dense factor in order: V_spd (32 x n), V_skh (32 x n).
Arithmetic runs in `dtype` (float64 by default, float32 for a bit-closer restatement of an fp32 reference run);
`grad_eps` is torch.finfo(G.dtype).eps of the gradient dtype the reference saw (psgd_pro.py:122).
"""
import numpy as np

K_SUBSPACE = 32                      # psgd_pro_fast.py:29, psgd_pro.py:19 (k=32)
F32_TINY = np.finfo(np.float32).tiny  # torch.finfo(float32).smallest_normal, psgd_pro.py:31


def _tiny(dtype):
    return np.finfo(dtype).tiny


def vector_norm_rows(V):
    return np.sqrt(np.sum(V * V, axis=1))


def _norm_lower_bound(A, nf, V, half_iters=2):
    """psgd_pro_fast.py:32-43 (psgd_pro.py:19-41 with the random start passed in): A / nf, the row of largest norm
    steers the 32 random vectors, 2 x (V A, row-normalise, V A), returns nf * max row norm."""
    tiny = _tiny(A.dtype)
    A = A / nf
    j = int(np.argmax(vector_norm_rows(A)))
    Aj = A[j:j + 1]
    V = Aj + np.sign(np.sum(Aj * V, axis=1, keepdims=True)) * V
    for _ in range(half_iters):
        V = V @ A
        V = V / (vector_norm_rows(V)[:, None] + tiny)
        V = V @ A
    return nf * np.max(vector_norm_rows(V))


def norm_lower_bound_spd(A, V):
    """psgd_pro_fast.py:46-47; psgd_pro.py:19-41 (normalising factor = max diagonal + smallest normal)."""
    return _norm_lower_bound(A, np.max(np.diagonal(A)) + _tiny(A.dtype), V)


def norm_lower_bound_skh(A, V):
    """psgd_pro_fast.py:50-51; psgd_pro.py:43-65 (normalising factor = max |A_ij| + smallest normal)."""
    return _norm_lower_bound(A, np.max(np.abs(A)) + _tiny(A.dtype), V)


def procrustes_step2(Q, V, max_step_size=1 / 8):
    """psgd_pro.py:71-94 (psgd_pro_fast.py:129-138): rotate Q by the 2nd-order expansion of exp(aR), R = Q^T - Q
    normalised by its norm lower bound, with the line search on a. Returns the new Q."""
    R = Q.T - Q
    R = R / (norm_lower_bound_skh(R, V) + _tiny(Q.dtype))
    RQ = R @ Q
    RRQ = R @ RQ
    tr_RQ = np.trace(RQ)
    tr_RRQ = np.trace(RRQ)
    a = min(-tr_RQ / tr_RRQ, max_step_size) if tr_RRQ < 0 else max_step_size
    return Q + a * (RQ + 0.5 * a * RRQ)


def procrustes_step_r2(Q, V, max_step_size=1 / 8):
    """psgd_pro_fast.py:141-153: the same rotation with Rn = Q - Q^T and S = Rn^T Rn (one symmetric product):
    tr(RQ) = sum(Rn * Q), tr(RRQ) = -sum(S * Q), Q - (a Rn + a^2/2 S) Q."""
    Rn = Q - Q.T
    Rn = Rn / (norm_lower_bound_skh(Rn, V) + _tiny(Q.dtype))
    S = Rn.T @ Rn
    tr_RQ = np.sum(Rn * Q)
    tr_RRQ = -np.sum(S * Q)
    a = min(-tr_RQ / tr_RRQ, max_step_size) if tr_RRQ < 0 else max_step_size
    return Q - (a * Rn + 0.5 * a * a * S) @ Q


def balance_kron_precond(Q):
    """psgd_pro.py:96-105: scale the factors to the geometric mean of their max-abs values (order > 1 only)."""
    if len(Q) <= 1:
        return Q
    norms = [np.max(np.abs(q)) for q in Q]
    gmean = np.prod(np.array(norms, dtype=np.float64)) ** (1.0 / len(Q))
    return [q * (gmean / nm) for q, nm in zip(Q, norms)]


def is_dense(size, numel, max_size, max_skew):
    """psgd_pro.py:189: a dim gets a diagonal factor if size <= 1, size > max_size or size^2 > max_skew * numel."""
    return not (size <= 1 or size > max_size or size ** 2 > max_skew * numel)


def init_kron(shape, scale, max_size=float("inf"), max_skew=1.0, dtype=np.float64):
    """psgd_pro.py:141-249 (dQ = Q0.5EQ1.5): per dim a dense scale^(1/order) I or a diagonal scale^(1/order) ones,
    L = 0 per factor (:181, :188, :191, :210). A 0-d tensor gets one scalar factor (:169-171)."""
    if len(shape) == 0:
        return [np.array(scale, dtype=dtype)], [0.0]
    numel = int(np.prod(shape))
    s = scale ** (1.0 / len(shape))
    Q = [s * np.eye(n, dtype=dtype) if is_dense(n, numel, max_size, max_skew) else s * np.ones(n, dtype=dtype)
         for n in shape]
    return Q, [0.0 for _ in shape]


def _mode_apply(X, M, i):
    """X x_i M: contracts mode i of X with the second index of M (M[a, b] X[.., b, ..])."""
    return np.moveaxis(np.tensordot(M, X, axes=([1], [i])), 0, i)


def precond_grad(Q, G):
    """psgd_pro.py:107-112 (exprP of :237-238): Pg = G x_1 P_1 x_2 P_2 ..., P_i = Q_i^T Q_i for a dense factor,
    q_i^2 along dim i for a diagonal one; a 0-d G is scaled by q^2."""
    if G.ndim == 0:
        return Q[0] * Q[0] * G
    Pg = G
    for i, q in enumerate(Q):
        if q.ndim == 2:
            Pg = _mode_apply(Pg, q.T @ q, i)
        else:
            shp = [1] * G.ndim
            shp[i] = -1
            Pg = Pg * (q * q).reshape(shp)
    return Pg


def _term1(Pg, i, dense):
    """exprGs[i](Pg, Pg) (psgd_pro.py:202-205 diagonal, :222-228 dense): contraction over every mode but i."""
    other = tuple(a for a in range(Pg.ndim) if a != i)
    if not dense:
        return np.sum(Pg * Pg, axis=other)
    X = np.moveaxis(Pg, i, 0).reshape(Pg.shape[i], -1)
    return X @ X.T


def update_precond(Q, L, G, rnd, lr=0.1, betaL=0.9, damping=1e-9, grad_eps=None, r2=False):
    """psgd_pro.py:114-139 / psgd_pro_fast.py:209-236 (without the balancing coin, drawn by the caller).
    rnd = [xi, (V_spd, V_skh) per dense factor]. Returns (new Q list, new L list, the noisy Pg)."""
    dtype = G.dtype
    eps = np.finfo(np.float32).eps if grad_eps is None else grad_eps
    rnd = iter(rnd)
    total = G.size
    damp = damping + eps * np.abs(G)
    Pg = precond_grad(Q, G + damp * next(rnd).astype(dtype))
    Qn, Ln = [], []
    for i, q in enumerate(Q):
        if q.ndim < 2:
            term1 = Pg * Pg if G.ndim == 0 else _term1(Pg, i, False)
            term2 = total / q.size
            ell = np.max(term1) + term2
            Li = max(betaL * L[i] + (1 - betaL) * ell, ell)
            Qn.append(q * (1 - lr / Li * (term1 - term2)))
        else:
            term1 = _term1(Pg, i, True)
            term2 = total / q.shape[0]
            ell = norm_lower_bound_spd(term1, next(rnd).astype(dtype)) + term2
            Li = max(betaL * L[i] + (1 - betaL) * ell, ell)
            qn = q - lr / Li * (term1 @ q - term2 * q)
            Vs = next(rnd).astype(dtype)
            qn = procrustes_step_r2(qn, Vs) if r2 else procrustes_step2(qn, Vs)
            Qn.append(qn)
        Ln.append(float(Li))
    return Qn, Ln, Pg


def clip_apply(param, Pg, lr, max_avg_amp=2.0, max_element_amp=10.0):
    """psgd_pro.py:371-381 (branch-free psgd_pro_fast.py:426-438): scale Pg to RMS <= max_avg_amp, clamp each
    element to +-max_element_amp, param -= lr * Pg."""
    avg = np.sqrt(np.mean(Pg * Pg))
    g = Pg * min(1.0, max_avg_amp / avg) if avg > 0 else Pg
    g = np.clip(g, -max_element_amp, max_element_amp)
    return param - lr * g.reshape(param.shape)


def draw_normals(rng, Q, shape):
    """The Gaussian draws of one update in the reference's order (psgd_pro_fast.py:200-206), float32."""
    out = [rng.standard_normal(shape, dtype=np.float32)]
    for q in Q:
        if q.ndim == 2:
            out += [rng.standard_normal((K_SUBSPACE, q.shape[0]), dtype=np.float32) for _ in range(2)]
    return out


class KronWhitenOracle:
    """psgd_pro.KronWhiten (psgd_pro.py:251-384) restated on numpy arrays, with every random draw supplied.

    step(grads, draws): draws = {"update": u, "coins": [c per param], "normals": [draw list per param]}; the update
    runs when u < preconditioner_update_probability (:345), balancing for a parameter when its coin < 0.01 (:138).
    Parameters are squeezed like the reference (:327) and updated in place of self.params (float arrays)."""

    def __init__(self, params, preconditioner_max_size=float("inf"), preconditioner_max_skew=1.0,
                 preconditioner_init_scale=None, lr_params=0.001, lr_preconditioner=0.1, betaL=0.9, damping=1e-9,
                 momentum=0.0, grad_clip_max_amps=(2.0, 10.0), preconditioner_update_probability=1.0,
                 update_preconditioner_first=True, whiten_grad=True, dtype=np.float64, grad_eps=None, r2=False):
        self.params = [np.array(p, dtype=dtype) for p in params]
        self.lr_params, self.lr_preconditioner, self.betaL, self.damping = lr_params, lr_preconditioner, betaL, damping
        self.momentum = momentum if 0 < momentum < 1 else 0.0
        self.grad_clip_max_amps = grad_clip_max_amps
        self.preconditioner_update_probability = preconditioner_update_probability
        self.update_preconditioner_first = update_preconditioner_first
        self.whiten_grad, self.dtype, self.grad_eps, self.r2 = whiten_grad, dtype, grad_eps, r2
        self.max_size, self.max_skew = preconditioner_max_size, preconditioner_max_skew
        self.QL = None
        if preconditioner_init_scale is not None:
            self.QL = [init_kron(np.squeeze(p).shape, preconditioner_init_scale, self.max_size, self.max_skew, dtype)
                       for p in self.params]
        self.ms, self.counter_m = None, 0

    def _init_on_the_fly(self, grads):
        """psgd_pro.py:329-332: scale = (max_i mean|g_i|^4 + damping^4)^(-1/8)."""
        scale = max(float(np.mean(np.abs(g) ** 4)) for g in grads)
        scale = (scale + self.damping ** 4) ** (-1 / 8)
        self.QL = [init_kron(g.shape, scale, self.max_size, self.max_skew, self.dtype) for g in grads]

    def _update(self, srcs, draws):
        for k, (QL, g) in enumerate(zip(self.QL, srcs)):
            Q, L, _ = update_precond(QL[0], QL[1], g, draws["normals"][k], self.lr_preconditioner, self.betaL,
                                     self.damping, self.grad_eps, self.r2)
            if draws["coins"][k] < 0.01:
                Q = balance_kron_precond(Q)
            self.QL[k] = (Q, L)

    def step(self, grads, draws):
        grads = [np.squeeze(np.asarray(g, dtype=self.dtype)) for g in grads]
        if self.QL is None:
            self._init_on_the_fly(grads)
        if self.momentum > 0:  # psgd_pro.py:334-343
            beta = min(self.counter_m / (1 + self.counter_m), self.momentum)
            self.counter_m += 1
            if self.ms is None:
                self.ms = [np.zeros_like(g) for g in grads]
            self.ms = [beta * m + (1 - beta) * g for m, g in zip(self.ms, grads)]
        else:
            self.ms, self.counter_m = None, 0
        update = draws["update"] < self.preconditioner_update_probability
        srcs = grads if self.whiten_grad else self.ms
        if update and self.update_preconditioner_first:
            self._update(srcs, draws)
        pre = [precond_grad(QL[0], m) for QL, m in zip(self.QL, self.ms if self.momentum > 0 else grads)]
        if update and not self.update_preconditioner_first:
            self._update(srcs, draws)
        a0, a1 = self.grad_clip_max_amps
        self.params = [clip_apply(p, g, self.lr_params, a0, a1) for p, g in zip(self.params, pre)]
        return pre

    def make_draws(self, rng, grads, coins=None):
        """Draws for one step from a numpy Generator, in the reference order."""
        grads = [np.squeeze(np.asarray(g)) for g in grads]
        if self.QL is None:
            self._init_on_the_fly([g.astype(self.dtype) for g in grads])
        u = float(rng.random(dtype=np.float32))
        c = [float(x) for x in rng.random(len(grads), dtype=np.float32)] if coins is None else list(coins)
        normals = [draw_normals(rng, QL[0], g.shape) for QL, g in zip(self.QL, grads)]
        return {"update": u, "coins": c, "normals": normals}
