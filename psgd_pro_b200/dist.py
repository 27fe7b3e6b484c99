"""Multi-GPU PSGD-Kron step: preconditioner blocks partitioned across ranks, updated parameters all-gathered.

Each parameter's preconditioner (its Q factors, L and preconditioned gradient) depends only on that parameter's
gradient (psgd_pro.py:352-361), so parameters are assigned whole to ranks by a longest-processing-time greedy on
their algorithmic FLOP count; every rank holds all (data-parallel reduced) gradients and all parameters, runs the
step for the parameters it owns, and the updated parameters are all-gathered (NCCL over NVLink) so that every
rank ends the step with the full parameter set. Q and L stay sharded.

Collectives: one all_gather_into_tensor per step over a flat buffer (in place when the parameters are views of
the flat layout make_flat_params builds, otherwise packed and unpacked around the collective)."""
import math

import torch
import torch.distributed as dist

K_SUB = 32


def _dense(size, numel, max_size, max_skew):
    return not (size <= 1 or size > max_size or size ** 2 > max_skew * numel)


def falg(shape, max_size=float("inf"), max_skew=1.0):
    """Algorithmic FLOPs of one step for a parameter of this (squeezed) shape: per 2-D dense factor of size n,
    6n^3 + 5nN + 512n^2; per 1-D dense factor 5n^3 + 521n^2; diagonal factors 0 (memory-bound)."""
    shape = [s for s in shape if s != 1]
    N = max(1, math.prod(shape))
    f = 0.0
    if len(shape) == 1:
        n = shape[0]
        if _dense(n, N, max_size, max_skew):
            f += 5 * n ** 3 + 521 * n ** 2
    elif len(shape) == 2:
        for n in shape:
            if _dense(n, N, max_size, max_skew):
                f += 6 * n ** 3 + 5 * n * N + 512 * n ** 2
    return f


def lpt_assign(costs, world):
    """Longest processing time first: each item (largest cost first) to the least-loaded rank. Returns the rank of
    each item; ties broken by rank index, so every process computes the same assignment."""
    load = [0.0] * world
    owner = [0] * len(costs)
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += costs[i]
    return owner


def assignment_for(shapes, world, max_size=float("inf"), max_skew=1.0, memory_weight=64.0):
    """Owner rank per parameter: FLOP cost plus a small per-element term so diagonal-only (memory-bound)
    parameters are spread as well."""
    costs = [falg(s, max_size, max_skew) + memory_weight * max(1, math.prod(s)) for s in shapes]
    return lpt_assign(costs, world)


def make_flat_params(shapes, owner, world, dtype, device, init=None):
    """Parameters as views of one flat buffer laid out rank by rank (segment r holds rank r's parameters, every
    segment padded to the same length), so the all-gather of the updated parameters needs no copies.
    Returns (params, flat, seg)."""
    sizes = [max(1, math.prod(s)) for s in shapes]
    per = [sum(sz for sz, o in zip(sizes, owner) if o == r) for r in range(world)]
    seg = max(per) if per else 0
    seg = (seg + 63) // 64 * 64
    flat = torch.zeros(world * seg, dtype=dtype, device=device)
    off = [r * seg for r in range(world)]
    params = []
    for s, sz, o in zip(shapes, sizes, owner):
        v = flat[off[o]:off[o] + sz].view(s)
        off[o] += sz
        if init is not None:
            v.copy_(init(s))
        params.append(torch.nn.Parameter(v, requires_grad=True))
    return params, flat, seg


class ShardedKronWhiten:
    """KronWhiten over a process group: this rank owns the parameters `assignment` gives it and runs the step for
    them; step_math(grads) takes the full gradient list (every rank's gradients are the same, as after a
    data-parallel all-reduce) and ends with every parameter updated on every rank.

    optimizer_factory(params, **kw) builds the per-rank optimizer (default psgd_pro_b200.KronWhiten); flat=(buffer,
    segment) marks parameters laid out by make_flat_params (in-place all-gather)."""

    def __init__(self, params, group=None, assignment=None, flat=None, optimizer_factory=None, **kw):
        self.params = list(params)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        shapes = [tuple(p.squeeze().shape) for p in self.params]
        self.owner = assignment if assignment is not None else assignment_for(
            shapes, self.world, kw.get("preconditioner_max_size", float("inf")),
            kw.get("preconditioner_max_skew", 1.0))
        self.owned = [i for i, o in enumerate(self.owner) if o == self.rank]
        if optimizer_factory is None:
            from .optimizer import KronWhiten
            optimizer_factory = KronWhiten
        self.opt = optimizer_factory([self.params[i] for i in self.owned], **kw) if self.owned else None
        self.flat = flat
        if flat is None and self.world > 1:
            sizes = [p.numel() for p in self.params]
            self._seg = max(sum(sz for sz, o in zip(sizes, self.owner) if o == r) for r in range(self.world))
            dt, dv = self.params[0].dtype, self.params[0].device
            self._send = torch.empty(self._seg, dtype=dt, device=dv)
            self._recv = torch.empty(self.world * self._seg, dtype=dt, device=dv)

    @property
    def inner(self):
        return self.opt

    @torch.no_grad()
    def step_math(self, grads, draws=None):
        """grads: one per parameter (all ranks pass the full list). draws (tests): the full draw set of
        KronWhiten.step_math; this rank keeps the coins and normals of its own parameters."""
        grads = list(grads)
        if draws is not None:
            draws = {"update": draws["update"], "coins": [draws["coins"][i] for i in self.owned] if draws["coins"] else [],
                     "normals": [draws["normals"][i] for i in self.owned] if draws["normals"] else []}
        if self.opt is not None:
            self.opt.step_math([grads[i] for i in self.owned], draws=draws)
        self.allgather()

    @torch.no_grad()
    def allgather(self):
        """Every rank receives the parameters updated by their owners."""
        if self.world == 1:
            return
        if self.flat is not None:
            buf, seg = self.flat
            dist.all_gather_into_tensor(buf, buf[self.rank * seg:(self.rank + 1) * seg], group=self.group)
            return
        off = 0
        for i in self.owned:
            n = self.params[i].numel()
            self._send[off:off + n].copy_(self.params[i].reshape(-1))
            off += n
        dist.all_gather_into_tensor(self._recv, self._send, group=self.group)
        offs = [r * self._seg for r in range(self.world)]
        for i, (p, o) in enumerate(zip(self.params, self.owner)):
            n = p.numel()
            if o != self.rank:
                p.view(-1).copy_(self._recv[offs[o]:offs[o] + n])
            offs[o] += n

    @torch.no_grad()
    def step(self, closure):
        with torch.enable_grad():
            closure_returns = closure()
            loss = closure_returns if isinstance(closure_returns, torch.Tensor) else closure_returns[0]
            grads = torch.autograd.grad(loss, self.params)
        self.step_math(grads)
        return closure_returns
