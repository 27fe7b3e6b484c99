"""Multi-GPU PSGD-Kron step: preconditioner blocks partitioned across ranks, updated parameters all-gathered.

Each parameter's preconditioner (its Q factors, L and preconditioned gradient) depends only on that parameter's
gradient (psgd_pro.py:352-361), so parameters are assigned whole to ranks by a longest-processing-time greedy on
their algorithmic FLOP count; every rank holds all (data-parallel reduced) gradients and all parameters, runs the
step for the parameters it owns, and the updated parameters are all-gathered (NCCL over NVLink) so that every
rank ends the step with the full parameter set. Q and L stay sharded.

Overlap: a rank's parameters are split into buckets (balanced by FLOPs, the bucket with the fewest bytes last), each
stepped by its own optimizer (one grouped launch per phase per bucket). When a bucket's step has been enqueued, its
all-gather (all_gather_into_tensor over that bucket's region of the flat parameter buffer, in place) starts on a
side stream, so it runs while the later buckets compute; only the last bucket's all-gather is exposed. The step
returns with the current stream waiting for every all-gather.

Reduce-scatter (reduce_scatter=True): the data-parallel gradient reduction is fused into the sharded step instead of
a separate all-reduce before it. Each rank passes its own local gradients; they sit in a flat buffer laid out like
the parameters, and per bucket one reduce_scatter_tensor (average over ranks) delivers to each rank the reduced
gradients of exactly the parameters it owns, which its optimizer then reads in place. All buckets' reduce-scatters
are issued at the start of the step on the side stream, so bucket b + 1's runs while bucket b computes."""
import math

import torch
import torch.distributed as dist

K_SUB = 32


def _dense(size, numel, max_size, max_skew):
    return not (size <= 1 or size > max_size or size ** 2 > max_skew * numel)


def falg(shape, max_size=float("inf"), max_skew=1.0):
    """Algorithmic FLOPs of one step for a parameter of this (squeezed) shape: per 2-D dense factor of size n,
    6n^3 + 5nN + 512n^2; per 1-D dense factor 5n^3 + 521n^2; diagonal factors 0 (memory-bound). An order-r
    parameter (r > 2) counts the same per dense factor: its factor work 6n^3 + 512n^2 and its share 5nN of the two
    preconditioner applications and term1."""
    shape = [s for s in shape if s != 1]
    N = max(1, math.prod(shape))
    f = 0.0
    if len(shape) == 1:
        n = shape[0]
        if _dense(n, N, max_size, max_skew):
            f += 5 * n ** 3 + 521 * n ** 2
    elif len(shape) >= 2:
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


def _cost(shape, max_size, max_skew, memory_weight=64.0):
    return falg(shape, max_size, max_skew) + memory_weight * max(1, math.prod(shape))


def assignment_for(shapes, world, max_size=float("inf"), max_skew=1.0, memory_weight=64.0):
    """Owner rank per parameter: FLOP cost plus a small per-element term so diagonal-only (memory-bound)
    parameters are spread as well."""
    return lpt_assign([_cost(s, max_size, max_skew, memory_weight) for s in shapes], world)


def bucket_assignment(shapes, owner, world, nbuckets, max_size=float("inf"), max_skew=1.0):
    """Bucket of each parameter within its owner's share: the owner's parameters are split by LPT on their cost
    into at most nbuckets buckets, which are then numbered by decreasing element count, so the last bucket (whose
    all-gather no later compute hides) moves the fewest bytes. Deterministic: every rank computes the same."""
    bucket = [0] * len(shapes)
    for r in range(world):
        idx = [i for i in range(len(shapes)) if owner[i] == r]
        if not idx:
            continue
        nb = max(1, min(nbuckets, len(idx)))
        sub = lpt_assign([_cost(shapes[i], max_size, max_skew) for i in idx], nb)
        sizes = [sum(max(1, math.prod(shapes[i])) for i, b in zip(idx, sub) if b == k) for k in range(nb)]
        order = sorted(range(nb), key=lambda k: (-sizes[k], k))
        rename = {k: j for j, k in enumerate(order)}
        for i, b in zip(idx, sub):
            bucket[i] = rename[b]
    return bucket


class FlatLayout:
    """Where each parameter lives in the flat buffer: bucket b occupies [start_b, start_b + world * seg_b), rank r's
    parameters of that bucket at start_b + r * seg_b onwards (every rank's share padded to seg_b elements), so the
    all-gather of a bucket is one in-place all_gather_into_tensor."""

    def __init__(self, shapes, owner, world, bucket):
        self.world, self.bucket_of = world, list(bucket)
        self.nbuckets = (max(bucket) + 1) if bucket else 1
        sizes = [max(1, math.prod(s)) for s in shapes]
        self.start, self.seg = [], []
        off = 0
        for b in range(self.nbuckets):
            per = [sum(sz for sz, o, bb in zip(sizes, owner, bucket) if o == r and bb == b) for r in range(world)]
            seg = (max(per) + 63) // 64 * 64 if per else 0
            self.start.append(off)
            self.seg.append(seg)
            off += world * seg
        self.total = off
        cursor = {(r, b): self.start[b] + r * self.seg[b] for r in range(world) for b in range(self.nbuckets)}
        self.offset = []
        for sz, o, b in zip(sizes, owner, bucket):
            self.offset.append(cursor[(o, b)])
            cursor[(o, b)] += sz


def make_flat_params(shapes, owner, world, dtype, device, init=None, buckets=None, max_size=float("inf"),
                     max_skew=1.0):
    """Parameters as views of one flat buffer laid out bucket by bucket and, inside a bucket, rank by rank (see
    FlatLayout), so the all-gathers of the updated parameters need no copies. buckets: per rank (default 1; the
    assignment is bucket_assignment's). Returns (params, flat, layout)."""
    nb = buckets or 1
    layout = FlatLayout(shapes, owner, world, bucket_assignment(shapes, owner, world, nb, max_size, max_skew))
    flat = torch.zeros(layout.total, dtype=dtype, device=device)
    params = []
    for s, off in zip(shapes, layout.offset):
        v = flat[off:off + max(1, math.prod(s))].view(s)
        if init is not None:
            v.copy_(init(s))
        params.append(torch.nn.Parameter(v, requires_grad=True))
    return params, flat, layout


class ShardedKronWhiten:
    """KronWhiten over a process group: this rank owns the parameters `assignment` gives it and runs the step for
    them; step_math(grads) takes the full gradient list (every rank's gradients are the same, as after a
    data-parallel all-reduce) and ends with every parameter updated on every rank.

    optimizer_factory(params, **kw) builds the per-bucket optimizer (default psgd_pro_b200.KronWhiten); flat=(buffer,
    layout) marks parameters laid out by make_flat_params (in-place all-gathers; the layout's buckets are used);
    buckets: all-gather buckets per rank when world > 1 (default 4; one when the parameters are not flat-laid);
    reduce_scatter: step_math takes each rank's local gradients and averages them over the ranks itself (see the
    module docstring); local_grads() gives views of the flat gradient buffer a training loop can fill in place."""

    def __init__(self, params, group=None, assignment=None, flat=None, optimizer_factory=None, buckets=None,
                 reduce_scatter=False, **kw):
        self.params = list(params)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        shapes = [tuple(p.squeeze().shape) for p in self.params]
        max_size, max_skew = kw.get("preconditioner_max_size", float("inf")), kw.get("preconditioner_max_skew", 1.0)
        self.owner = assignment if assignment is not None else assignment_for(shapes, self.world, max_size, max_skew)
        if flat is not None and not isinstance(flat[1], FlatLayout):  # (buffer, segment): one bucket
            seg = flat[1]
            lay = FlatLayout([tuple(p.shape) for p in self.params], self.owner, self.world, [0] * len(self.params))
            assert lay.seg[0] <= seg, "flat segment smaller than a rank's parameters"
            lay.seg = [seg]
            flat = (flat[0], lay)
        if flat is not None:
            self.bucket_of = flat[1].bucket_of
        elif self.world > 1:
            self.bucket_of = bucket_assignment(shapes, self.owner, self.world, buckets or 1, max_size, max_skew)
        else:
            self.bucket_of = [0] * len(self.params)
        self.nbuckets = (max(self.bucket_of) + 1) if self.bucket_of else 1
        self.members = [[i for i, (o, b) in enumerate(zip(self.owner, self.bucket_of)) if o == self.rank and b == k]
                        for k in range(self.nbuckets)]
        self.owned = [i for m in self.members for i in m]
        if optimizer_factory is None:
            from .optimizer import KronWhiten
            optimizer_factory = KronWhiten
        self.opts = [optimizer_factory([self.params[i] for i in m], **kw) if m else None for m in self.members]
        # With no preconditioner_init_scale the scale comes from the first gradients: the maximum of mean|g|^4 over
        # ALL parameters (psgd_pro.py:329-332), which every rank can take since every rank holds every gradient.
        self._scale_pending = kw.get("preconditioner_init_scale") is None
        self._damping = kw.get("damping", 1e-9)
        self.flat = flat
        self._side = None
        self.timing = None  # a list: each step appends its CUDA events (timing_ms() reads them)
        self.rs = bool(reduce_scatter) and self.world > 1
        self.rs_consumed = None
        if self.rs:
            lay = flat[1] if flat is not None else FlatLayout([tuple(p.shape) for p in self.params], self.owner,
                                                              self.world, self.bucket_of)
            self._glay = lay
            dt, dv = self.params[0].dtype, self.params[0].device
            self._gflat = torch.zeros(lay.total, dtype=dt, device=dv)  # local gradients, parameter layout
            self._gviews = [self._gflat[o:o + p.numel()].view(p.shape) for o, p in zip(lay.offset, self.params)]
            # this rank's reduced gradients: bucket b's chunk at gown_off[b], the owned parameters in layout order
            self._gown_off, off = [], 0
            for k in range(self.nbuckets):
                self._gown_off.append(off)
                off += lay.seg[k]
            self._gown = torch.zeros(max(1, off), dtype=dt, device=dv)
            self._gred = {}
            for i, (o, b) in enumerate(zip(self.owner, self.bucket_of)):
                if o == self.rank:
                    start = self._gown_off[b] + (lay.offset[i] - lay.start[b] - self.rank * lay.seg[b])
                    self._gred[i] = self._gown[start:start + self.params[i].numel()].view(self.params[i].shape)
        if flat is None and self.world > 1:
            sizes = [p.numel() for p in self.params]
            self._seg = [max(sum(sz for sz, o, b in zip(sizes, self.owner, self.bucket_of) if o == r and b == k)
                             for r in range(self.world)) for k in range(self.nbuckets)]
            dt, dv = self.params[0].dtype, self.params[0].device
            self._send = [torch.empty(max(1, s), dtype=dt, device=dv) for s in self._seg]
            self._recv = [torch.empty(self.world * max(1, s), dtype=dt, device=dv) for s in self._seg]

    @property
    def inner(self):
        """The first of this rank's per-bucket optimizers (the only one when world == 1)."""
        return next((o for o in self.opts if o is not None), None)

    @property
    def inners(self):
        return [o for o in self.opts if o is not None]

    def gather_bytes(self):
        """Bytes each rank receives per step over all buckets."""
        if self.world == 1:
            return 0
        el = self.params[0].element_size()
        segs = self.flat[1].seg if self.flat is not None else self._seg
        return sum((self.world - 1) * s * el for s in segs)

    def local_grads(self):
        """reduce_scatter mode: views of the flat local-gradient buffer, one per parameter (shaped like it). A loop
        that writes its gradients there (or passes these views to step_math) saves the packing copy."""
        return list(self._gviews) if self.rs else None

    def clip_scales_into(self, host):
        """Copies the per-parameter clip scales of the last step (this rank's parameters, bucket order) into a
        pinned host tensor without waiting (the step's metric)."""
        off = 0
        for o in self.inners:
            n = len(o._plan.params)
            host[off:off + n].copy_(o._plan.clip[:n], non_blocking=True)
            off += n

    @torch.no_grad()
    def step_math(self, grads, draws=None):
        """grads: one per parameter (all ranks pass the full list). draws (tests): the full draw set of
        KronWhiten.step_math; each bucket keeps the coins and normals of its own parameters."""
        grads = list(grads)
        main = torch.cuda.current_stream() if self.world > 1 and self.params[0].is_cuda else None
        ev = None
        if self.timing is not None and main is not None:
            ev = {"start": torch.cuda.Event(enable_timing=True), "gather": []}
            ev["start"].record(main)
        rs_done = self._reduce_scatter(grads, main) if self.rs else None
        if self._scale_pending:
            from .optimizer import init_scale_from_grads
            if self.rs:  # the reduced gradients of this rank's parameters, then the maximum over the ranks
                for e in rs_done:
                    if e is not None:
                        main.wait_event(e)
                own = [self._gred[i] for m in self.members for i in m]
                m4 = 0.0 if not own else max(float(torch.mean(g.to(torch.float64).abs() ** 4)) for g in own)
                t = torch.tensor([m4], dtype=torch.float64, device=self.params[0].device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
                scale = (float(t.item()) + self._damping ** 4) ** (-1 / 8)
            else:
                scale = init_scale_from_grads(grads, self._damping)
            for o in self.inners:
                o.set_init_scale(scale)
            self._scale_pending = False
        for k, (m, o) in enumerate(zip(self.members, self.opts)):
            if o is not None:
                d = None
                if draws is not None:
                    d = {"update": draws["update"],
                         "coins": [draws["coins"][i] for i in m] if draws["coins"] else [],
                         "normals": [draws["normals"][i] for i in m] if draws["normals"] else []}
                if self.rs:
                    if rs_done[k] is not None:
                        main.wait_event(rs_done[k])
                    g = [self._gred[i] for i in m]
                else:
                    g = [grads[i] for i in m]
                o.step_math(g, draws=d)
            self._allgather(k, main, ev)
        if main is not None:
            if ev is not None:
                ev["compute_end"] = torch.cuda.Event(enable_timing=True)
                ev["compute_end"].record(main)
            main.wait_stream(self._side)
            if ev is not None:
                ev["end"] = torch.cuda.Event(enable_timing=True)
                ev["end"].record(main)
                self.timing.append(ev)

    def _reduce_scatter(self, grads, main):
        """Packs the local gradients into the flat buffer (unless they are its views already) and issues every
        bucket's reduce-scatter (average over the ranks) on the side stream; returns an event per bucket."""
        for g, v in zip(grads, self._gviews):
            if g.data_ptr() != v.data_ptr():
                v.copy_(g.reshape(v.shape))
        lay = self._glay
        avg = dist.get_backend(self.group) == "nccl"
        if main is None:  # CPU tensors (gloo): synchronous
            for k in range(self.nbuckets):
                self._rs_bucket(k, lay, avg)
            return [None] * self.nbuckets
        if self._side is None:
            self._side = torch.cuda.Stream(self.params[0].device)
        self._side.wait_stream(main)
        done = []
        with torch.cuda.stream(self._side):
            for k in range(self.nbuckets):
                self._rs_bucket(k, lay, avg)
                e = torch.cuda.Event()
                e.record(self._side)
                done.append(e)
        self.rs_consumed = done[-1]  # the local-gradient buffer may be refilled once this event has completed
        return done

    def _rs_bucket(self, k, lay, avg):
        s, seg = lay.start[k], lay.seg[k]
        out = self._gown[self._gown_off[k]:self._gown_off[k] + seg]
        region = self._gflat[s:s + self.world * seg]
        if avg:
            dist.reduce_scatter_tensor(out, region, op=dist.ReduceOp.AVG, group=self.group)
        else:  # gloo has no average: sum, then scale
            dist.reduce_scatter_tensor(out, region, op=dist.ReduceOp.SUM, group=self.group)
            out.mul_(1.0 / self.world)

    def timing_ms(self):
        """Per recorded step (after a synchronize): compute_ms (start to the end of the last bucket's step),
        gather_ms (sum of the all-gathers' durations) and exposed_gather_ms (end of compute to end of step)."""
        out = []
        for ev in self.timing or []:
            out.append({"compute_ms": ev["start"].elapsed_time(ev["compute_end"]),
                        "gather_ms": sum(a.elapsed_time(b) for a, b in ev["gather"]),
                        "exposed_gather_ms": max(0.0, ev["compute_end"].elapsed_time(ev["end"]))})
        return out

    @torch.no_grad()
    def _allgather(self, k, main, ev):
        """Bucket k's all-gather, on the side stream once the bucket's step has been enqueued on the current one."""
        if self.world == 1:
            return
        if main is None:  # CPU tensors (gloo): synchronous
            self._gather_bucket(k)
            return
        if self._side is None:
            self._side = torch.cuda.Stream(self.params[0].device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            if ev is not None:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(self._side)
            self._gather_bucket(k)
            if ev is not None:
                b.record(self._side)
                ev["gather"].append((a, b))

    def _gather_bucket(self, k):
        if self.flat is not None:
            buf, lay = self.flat
            s, seg = lay.start[k], lay.seg[k]
            region = buf[s:s + self.world * seg]
            dist.all_gather_into_tensor(region, region[self.rank * seg:(self.rank + 1) * seg], group=self.group)
            return
        send, recv, seg = self._send[k], self._recv[k], max(1, self._seg[k])
        off = 0
        for i in self.members[k]:
            n = self.params[i].numel()
            send[off:off + n].copy_(self.params[i].reshape(-1))
            off += n
        dist.all_gather_into_tensor(recv, send, group=self.group)
        offs = [r * seg for r in range(self.world)]
        for i, (p, o, b) in enumerate(zip(self.params, self.owner, self.bucket_of)):
            if b != k:
                continue
            n = p.numel()
            if o != self.rank:
                p.view(-1).copy_(recv[offs[o]:offs[o] + n])
            offs[o] += n

    @torch.no_grad()
    def step(self, closure):
        with torch.enable_grad():
            closure_returns = closure()
            loss = closure_returns if isinstance(closure_returns, torch.Tensor) else closure_returns[0]
            grads = torch.autograd.grad(loss, self.params)
        self.step_math(grads)
        return closure_returns
