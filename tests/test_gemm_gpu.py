"""tcgen05 GEMM (libpsgd_b200.so, psgd_gemm / psgd_gemm_launch) against plain PyTorch fp32/fp64 products of the
same operands: plain and split (hi/lo) arithmetic, SYRK with mirrored output, the fused epilogue terms and
reductions, and grouped launches over problems of different shapes."""
import pytest
import torch

from psgd_pro_b200 import kernels as K

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def bf16_operand(rows, cols, dev, gen, split=False, scale=1.0):
    x = torch.randn(rows, cols, generator=gen, device="cpu").mul_(scale).to(dev)
    hi, lo = K.operand(rows, cols, dev, split=split)
    K.split_into(x, hi, lo)
    return x, (hi, lo)


def err_word(dev):
    return torch.zeros(1, dtype=torch.int32, device=dev)


@pytest.mark.parametrize("M,N,Kd,bn", [(128, 128, 64, 128), (256, 512, 1024, 256), (200, 72, 100, 64),
                                       (1, 16, 8, 16), (300, 33, 70, 32), (130, 260, 129, 256)])
def test_plain_bf16(cuda, M, N, Kd, bn):
    g = torch.Generator().manual_seed(M * 7 + N)
    a, A = bf16_operand(M, Kd, cuda, g)
    b, B = bf16_operand(N, Kd, cuda, g)
    out = torch.full((M, N), float("nan"), device=cuda)
    err = err_word(cuda)
    K.gemm(K.make_spec(A, B, M, N, Kd, bn=bn, out_f32=out), 1, err)
    ref = A[0][:, :Kd].float() @ B[0][:, :Kd].float().T
    torch.cuda.synchronize()
    assert err.item() == 0
    assert rel(out, ref) < 1e-5


@pytest.mark.parametrize("M,N,Kd,bn", [(256, 256, 512, 128), (192, 576, 192, 64), (65, 10, 65, 16)])
def test_split_fp32(cuda, M, N, Kd, bn):
    g = torch.Generator().manual_seed(3)
    a, A = bf16_operand(M, Kd, cuda, g, split=True)
    b, B = bf16_operand(N, Kd, cuda, g, split=True)
    out = torch.empty(M, N, device=cuda)
    err = err_word(cuda)
    K.gemm(K.make_spec(A, B, M, N, Kd, bn=bn, out_f32=out), 3, err)
    ref = a.double() @ b.double().T
    torch.cuda.synchronize()
    assert err.item() == 0
    assert rel(out, ref) < 2e-5, rel(out, ref)
    # single-pass bf16 is visibly worse on the same inputs (the split is doing work)
    out1 = torch.empty(M, N, device=cuda)
    K.gemm(K.make_spec(A, B, M, N, Kd, bn=bn, out_f32=out1), 1, err)
    assert rel(out1, ref) > 10 * rel(out, ref)


@pytest.mark.parametrize("n,Kd,split,bn", [(128, 64, 1, 128), (384, 200, 3, 128), (300, 1000, 1, 128),
                                          (10, 7, 3, 128), (600, 300, 1, 256), (1030, 64, 1, 256), (256, 96, 1, 256),
                                          (512, 256, 1, 256), (768, 128, 3, 128), (1024, 64, 1, 256)])
def test_syrk_symmetric(cuda, n, Kd, split, bn):
    g = torch.Generator().manual_seed(n)
    x, X = bf16_operand(n, Kd, cuda, g, split=split == 3)
    Tm, Tn = (n + 127) // 128, (n + bn - 1) // bn
    out = torch.full((n, n), float("nan"), device=cuda)
    hi, lo = K.operand(n, n, cuda, split=split == 3)
    part_row = torch.zeros(Tn + Tm, n, device=cuda)  # zero once: slots no tile reaches stay zero
    diag = torch.empty(n, device=cuda)
    dot_aux = torch.randn(n, n, generator=g).to(cuda)
    part_dot = torch.zeros(Tm * Tn, device=cuda)
    err = err_word(cuda)
    spec = K.make_spec(X, X, n, n, Kd, bn=bn, mode=K.PSGD_GEMM_SYRK, out_f32=out, out_hi=hi, out_lo=lo,
                       part_row=part_row, diag_out=diag, dot_aux=dot_aux, part_dot=part_dot)
    K.gemm(spec, split, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    xs = x.double() if split == 3 else X[0][:, :Kd].double()
    ref = xs @ xs.T
    assert torch.equal(out, out.T)  # exactly symmetric
    assert rel(out, ref) < (2e-5 if split == 3 else 1e-5)
    assert rel(hi[:, :n].float(), ref) < 1e-2
    assert rel(part_row.sum(0), (ref ** 2).sum(1)) < 1e-4
    assert rel(diag, ref.diagonal()) < 2e-5
    got_dot = part_dot.double().sum().item()
    want = (ref * dot_aux.double()).sum().item()
    assert abs(got_dot - want) <= 1e-4 * (ref.abs() * dot_aux.double().abs()).sum().item()


def test_epilogue_terms(cuda):
    g = torch.Generator().manual_seed(11)
    M, N, Kd = 260, 96, 130
    a, A = bf16_operand(M, Kd, cuda, g, split=True)
    b, B = bf16_operand(N, Kd, cuda, g, split=True)
    aux = torch.randn(M, N, generator=g).to(cuda)
    rs = torch.rand(M, generator=g).to(cuda) + 0.5
    csv = torch.rand(N, generator=g).to(cuda) + 0.5
    ap = torch.tensor([0.25], device=cuda)
    bp = torch.tensor([2.0], device=cuda)
    out = torch.empty(M, N, device=cuda)
    hi_t, lo_t = K.operand(N, M, cuda, split=True)
    tm_n, tn_n = (M + 127) // 128, (N + 31) // 32
    part_tile = torch.zeros(tm_n * tn_n, device=cuda)
    part_col = torch.zeros(tm_n, N, device=cuda)
    part_row = torch.zeros(tn_n, M, device=cuda)
    err = err_word(cuda)
    spec = K.make_spec(A, B, M, N, Kd, bn=32, alpha=-3.0, beta=0.5, alpha_ptr=ap, beta_ptr=bp, aux=aux, row_scale=rs,
                       col_scale=csv, out_f32=out, out_hi_t=hi_t, out_lo_t=lo_t, part_tile=part_tile,
                       part_col=part_col, part_row=part_row)
    K.gemm(spec, 3, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = ((-0.75) * (a.double() @ b.double().T) + 1.0 * aux.double()) * rs.double()[:, None] * csv.double()[None, :]
    assert rel(out, ref) < 2e-5
    assert rel(hi_t[:, :M].float() + lo_t[:, :M].float(), ref.T) < 2e-5
    assert rel(part_tile.sum(), (ref ** 2).sum()) < 1e-5
    assert rel(part_col.sum(0), (ref ** 2).sum(0)) < 1e-5
    assert rel(part_row.sum(0), (ref ** 2).sum(1)) < 1e-5


def test_col_scale_from_partials(cuda):
    """cs_mode 2: column c scaled by 1 / (nf (||prev_c|| + tiny)) from a previous product's column partials."""
    g = torch.Generator().manual_seed(5)
    M, N, Kd = 384, 32, 384
    a, A = bf16_operand(M, Kd, cuda, g)
    b, B = bf16_operand(N, Kd, cuda, g)
    T = 3
    parts = torch.rand(T, N, generator=g).to(cuda)
    nf = torch.tensor([1.7], device=cuda)
    out = torch.empty(M, N, device=cuda)
    err = err_word(cuda)
    K.gemm(K.make_spec(A, B, M, N, Kd, bn=32, out_f32=out, cs_part=parts, cs_T=T, cs_mode=2, cs_nf=nf), 1, err)
    torch.cuda.synchronize()
    sc = 1.0 / (1.7 * (parts.double().sum(0).sqrt() + torch.finfo(torch.float32).tiny))
    ref = (A[0][:, :Kd].double() @ B[0][:, :Kd].double().T) * sc[None, :]
    assert rel(out, ref) < 1e-5


@pytest.mark.parametrize("split", [1, 3])
def test_group_launch(cuda, split):
    g = torch.Generator().manual_seed(17)
    shapes = [(512, 512, 512, 128), (64, 10, 64, 16), (300, 700, 90, 64), (1024, 256, 256, 128), (8, 8, 8, 16)]
    if split == 1:
        shapes.append((640, 512, 320, 256))
    specs, refs, outs, keep = [], [], [], []
    for (M, N, Kd, bn) in shapes:
        a, A = bf16_operand(M, Kd, cuda, g, split=split == 3)
        b, B = bf16_operand(N, Kd, cuda, g, split=split == 3)
        keep += [A, B]  # specs hold raw device pointers: the operands must outlive the launches
        out = torch.empty(M, N, device=cuda)
        specs.append(K.make_spec(A, B, M, N, Kd, bn=bn, out_f32=out))
        outs.append(out)
        refs.append(a.double() @ b.double().T if split == 3 else A[0][:, :Kd].double() @ B[0][:, :Kd].double().T)
    n = 48
    x, X = bf16_operand(n, 100, cuda, g, split=split == 3)
    sy = torch.empty(n, n, device=cuda)
    specs.append(K.make_spec(X, X, n, n, 100, bn=128, mode=K.PSGD_GEMM_SYRK, out_f32=sy))
    xs = x.double() if split == 3 else X[0][:, :100].double()
    outs.append(sy)
    refs.append(xs @ xs.T)
    keep.append(X)
    grp = K.GemmGroup(specs, split, cuda, keep=keep)
    err = err_word(cuda)
    for _ in range(3):  # relaunch: same results
        grp.launch(err)
    torch.cuda.synchronize()
    assert err.item() == 0
    for o, r in zip(outs, refs):
        assert rel(o, r) < (2e-5 if split == 3 else 1e-5)


def _pair_group(cuda, build, pair, monkeypatch):
    """The same problems encoded for the pair kernel (tcgen05 cta_group::2) or, with PSGD_GEMM_PAIR=0, for the
    one-CTA kernel; returns the outputs after two launches."""
    monkeypatch.setenv("PSGD_GEMM_PAIR", "1" if pair else "0")
    specs, outs, keep = build()
    grp = K.GemmGroup(specs, 1, cuda, keep=keep)
    assert bool(grp.kind & 8) == pair
    err = err_word(cuda)
    grp.launch(err)
    grp.launch(err)
    torch.cuda.synchronize()
    assert err.item() == 0
    return outs


def test_pair_kernel_plain_and_transposed(cuda, monkeypatch):
    g = torch.Generator().manual_seed(23)
    shapes = [(512, 512, 320, 256), (768, 1024, 200, 256), (256, 256, 64, 256), (768, 384, 128, 128),
              (1280, 2560, 1000, 256), (400, 400, 77, 256)]  # the last one: partial pair tiles on both edges
    data = [(bf16_operand(M, Kd, cuda, g), bf16_operand(N, Kd, cuda, g)) for (M, N, Kd, bn) in shapes]

    def build():
        specs, outs, keep = [], [], []
        for (M, N, Kd, bn), ((a, A), (b, B)) in zip(shapes, data):
            out = torch.full((M, N), float("nan"), device=cuda)
            ht = K.operand(N, M, cuda, split=False)
            keep += [A, B, ht]
            specs.append(K.make_spec(A, B, M, N, Kd, bn=bn, out_f32=out, out_hi_t=ht[0]))
            outs.append((out, ht[0]))
        return specs, outs, keep

    pair = _pair_group(cuda, build, True, monkeypatch)
    single = _pair_group(cuda, build, False, monkeypatch)
    for (M, N, Kd, bn), ((a, A), (b, B)), (o, t), (o1, t1) in zip(shapes, data, pair, single):
        ref = A[0][:, :Kd].double() @ B[0][:, :Kd].double().T
        assert rel(o, ref) < 1e-5, (M, N)
        assert rel(o, o1) < 1e-6
        assert rel(t[:, :M].float(), ref.T) < 1e-2


@pytest.mark.parametrize("dot", [True, False])
def test_pair_kernel_syrk_reductions(cuda, monkeypatch, dot):
    """SYRK on CTA pairs and on one CTA: fp32 and bf16 outputs (both triangles, the mirror through TMA stores on
    pairs), row sums of squares and the diagonal; with the trace operand (dot) the tiles take the general epilogue,
    without it the fast one."""
    g = torch.Generator().manual_seed(29)
    cases = [(512, 96), (768, 300), (1280, 64), (2048, 512)]
    data = [bf16_operand(n, Kd, cuda, g) for n, Kd in cases]
    qs = [torch.randn(n, n, generator=g).to(cuda) for n, _ in cases]

    def build():
        specs, outs, keep = [], [], []
        for (n, Kd), (x, X), q in zip(cases, data, qs):
            Tm, Tn = (n + 127) // 128, (n + 255) // 256
            out = torch.full((n, n), float("nan"), device=cuda)
            hi = K.operand(n, n, cuda, split=False)
            part_row = torch.zeros(Tn + Tm, n, device=cuda)
            diag = torch.empty(n, device=cuda)
            part_dot = torch.zeros(Tm * Tn, device=cuda)
            keep += [X, hi]
            extra = dict(dot_aux=q, part_dot=part_dot) if dot else {}
            specs.append(K.make_spec(X, X, n, n, Kd, bn=256, mode=K.PSGD_GEMM_SYRK, out_f32=out, out_hi=hi[0],
                                     part_row=part_row, diag_out=diag, **extra))
            outs.append((out, hi[0], part_row, diag, part_dot))
        return specs, outs, keep

    for pair in (True, False):
        for (n, Kd), (x, X), q, (out, hi, part_row, diag, part_dot) in zip(
                cases, data, qs, _pair_group(cuda, build, pair, monkeypatch)):
            ref = X[0][:, :Kd].double() @ X[0][:, :Kd].double().T
            assert torch.equal(out, out.T), (n, pair)
            assert rel(out, ref) < 1e-5
            h = hi[:, :n]
            assert torch.equal(h, h.T), (n, pair)
            assert rel(h.float(), ref) < 1e-2
            assert rel(part_row.sum(0), (ref ** 2).sum(1)) < 1e-4
            assert rel(diag, ref.diagonal()) < 2e-5
            if dot:
                want = (ref * q.double()).sum().item()
                assert abs(part_dot.double().sum().item() - want) <= \
                    1e-4 * (ref.abs() * q.double().abs()).sum().item()


def bf16_operand_from(x, dev):
    hi, lo = K.operand(x.shape[0], x.shape[1], dev, split=False)
    K.split_into(x.to(dev), hi, lo)
    return x, (hi, lo)


def test_pair_kernel_trmm(cuda, monkeypatch):
    """TRMM mode on CTA pairs: C = triu(T) X. The operand holds zeros below the diagonal inside each tile's diagonal
    band and NaN in the blocks left of it (columns before the tile's first row, 256-row tiles), which the K loop must
    never read (K-block counts even and odd, pair tiles partial at the edge)."""
    g = torch.Generator().manual_seed(37)
    cases = [(512, 256), (1024, 512), (768, 512), (1000, 256)]
    data = []
    for n, p in cases:
        T = torch.triu(torch.randn(n, n, generator=g) / n ** 0.5)
        x = torch.randn(p, n, generator=g)  # X^T: the K-major operand of the product
        i = torch.arange(n).view(n, 1)
        j = torch.arange(n).view(1, n)
        Tp = T.masked_fill(j < 256 * (i // 256), float("nan"))
        (_, Top), (_, Xop) = bf16_operand_from(Tp, cuda), bf16_operand_from(x, cuda)
        data.append((T, x, Top, Xop))

    def build():
        specs, outs, keep = [], [], []
        for (n, p), (_, _, Top, Xop) in zip(cases, data):
            out = torch.full((n, p), float("nan"), device=cuda)
            keep += [Top, Xop]
            specs.append(K.make_spec(Top, Xop, n, p, n, bn=256, mode=K.PSGD_GEMM_TRMM, out_f32=out))
            outs.append(out)
        return specs, outs, keep

    pair = _pair_group(cuda, build, True, monkeypatch)
    single = _pair_group(cuda, build, False, monkeypatch)
    for (n, p), (Tu, x, Top, Xop), o, o1 in zip(cases, data, pair, single):
        ref = Top[0][:, :n].float().nan_to_num(0.0).double() @ Xop[0][:, :n].double().T
        assert torch.isfinite(o).all(), (n, p)
        assert rel(o, ref) < 1e-5, (n, p)
        assert rel(o, o1) < 1e-6


def test_pair_kernel_aux_epilogue(cuda, monkeypatch):
    """The q-update form: Q <- beta Q + alpha (A B^T) with device scalars, Q^T stored as bf16."""
    g = torch.Generator().manual_seed(31)
    n = 1024
    (a, A), (b, B) = bf16_operand(n, n, cuda, g), bf16_operand(n, n, cuda, g, scale=0.01)
    q0 = torch.randn(n, n, generator=g).to(cuda)
    alpha = torch.tensor([-0.05], device=cuda)

    def build():
        q = q0.clone()
        qt = K.operand(n, n, cuda, split=False)
        spec = K.make_spec(A, B, n, n, n, bn=256, alpha_ptr=alpha, alpha=1.0, beta=1.0, aux=q, out_f32=q,
                           out_hi_t=qt[0])
        return [spec], [(q, qt[0])], [A, B, qt, q]

    (q, qt), = _pair_group(cuda, build, True, monkeypatch)
    (q1, _), = _pair_group(cuda, build, False, monkeypatch)
    step = A[0][:, :n].double() @ B[0][:, :n].double().T
    ref = q0.double() + 2 * (-0.05) * step  # two launches, the second on the first's output
    assert rel(q, ref) < 1e-5
    assert rel(q, q1) < 1e-6
    assert rel(qt[:, :n].float(), q.T) < 1e-2


def test_narrow_group_long_stages(cuda):
    """Groups whose tiles are all at most 64 wide run on the narrow configuration (four 64-deep K blocks per stage):
    K that ends inside a stage, K = 1, and every narrow width."""
    g = torch.Generator().manual_seed(43)
    shapes = [(512, 32, 1000, 32), (300, 10, 65, 16), (1024, 64, 300, 64), (128, 32, 1, 32), (700, 48, 257, 64)]
    specs, refs, outs, keep = [], [], [], []
    for (M, N, Kd, bn) in shapes:
        a, A = bf16_operand(M, Kd, cuda, g)
        b, B = bf16_operand(N, Kd, cuda, g)
        keep += [A, B]
        out = torch.full((M, N), float("nan"), device=cuda)
        specs.append(K.make_spec(A, B, M, N, Kd, bn=bn, out_f32=out))
        outs.append(out)
        refs.append(A[0][:, :Kd].double() @ B[0][:, :Kd].double().T)
    grp = K.GemmGroup(specs, 1, cuda, keep=keep)
    assert grp.kind & 16  # the narrow configuration
    err = err_word(cuda)
    grp.launch(err)
    grp.launch(err)
    torch.cuda.synchronize()
    assert err.item() == 0
    for o, r in zip(outs, refs):
        assert rel(o, r) < 1e-5
