"""Kernel-level parity on the GPU: each C-ABI kernel against the CPU oracle.

Tolerances: exact-fp32 kernels (SIMT GEMM, elementwise, reductions) 1e-5
relative; TF32 tensor-core GEMM 2e-3 relative to the output's scale (operands
rounded to 10-bit mantissas, fp32 accumulation); the optimizer is bit-exact.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tx():
    import tynx_b200 as tx

    return tx


def _rel(a, b):
    scale = max(float(np.abs(b).max()), 1e-30)
    return float(np.abs(a - b).max()) / scale


def _gemm(tx, A, B, ta, tb, math, *, alpha=1.0, beta=0.0, C0=None, bias=None, act="none"):
    from tynx_b200 import _core

    ctx = _core.context()
    ctx.math = math
    try:
        M = A.shape[1] if ta else A.shape[0]
        K = A.shape[0] if ta else A.shape[1]
        N = B.shape[0] if tb else B.shape[1]
        a = tx.Tensor(A)
        b = tx.Tensor(B)
        c = tx.Tensor(C0 if C0 is not None else np.zeros((M, N), np.float32))
        bb = tx.Tensor(bias) if bias is not None else None
        _core.gemm(ctx, M, N, K, a.ptr, A.shape[1], ta, b.ptr, B.shape[1], tb, c.ptr, N,
                   alpha=alpha, beta=beta, bias=bb.ptr if bb is not None else None, act=act)
        return c.numpy()
    finally:
        ctx.math = "tf32"


SHAPES = [
    (128, 128, 64), (256, 384, 256), (300, 200, 100), (4096, 1024, 784), (512, 10, 1024),
    (1024, 1024, 4096), (64, 256, 32), (1000, 64, 72), (16384, 28, 32), (10, 1024, 4096),
]


@pytest.mark.parametrize("math,tol", [("fp32", 1e-5), ("tf32", 2e-3), ("3xtf32", 1e-5),
                                      ("tf32trunc", 4e-3)])
@pytest.mark.parametrize("ta,tb", [(0, 1), (0, 0), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_matches_fp64(tx, math, tol, ta, tb, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    want = (A.T if ta else A).astype(np.float64) @ (B.T if tb else B).astype(np.float64)
    got = _gemm(tx, A, B, ta, tb, math)
    assert _rel(got, want) < tol


@pytest.mark.parametrize("math,tol", [("fp32", 1e-5), ("tf32", 3e-3)])
@pytest.mark.parametrize("act", ["none", "relu", "tanh", "gelu"])
def test_gemm_epilogue(tx, math, tol, act):
    from oracle import flex_oracle as fo

    rng = np.random.default_rng(5)
    M, N, K = 512, 384, 256
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32) * 0.1
    bias = rng.standard_normal(N).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    z = A.astype(np.float64) @ W.T.astype(np.float64) + bias + 0.5 * C0
    fn = {"none": lambda v: v, "relu": lambda v: np.maximum(v, 0), "tanh": np.tanh,
          "gelu": lambda v: fo.gelu(fo.T(v.astype(np.float32))).data}[act]
    got = _gemm(tx, A, W, 0, 1, math, beta=0.5, C0=C0, bias=bias, act=act)
    # errors are relative to the pre-activation scale: the contraction's rounding
    # is what the tolerance bounds, and act is 1-Lipschitz for all four choices
    assert float(np.abs(got - fn(z)).max()) < tol * float(np.abs(z).max())


def _np_act(act, v):
    from scipy.special import erf

    return {"none": lambda x: x, "relu": lambda x: np.maximum(x, 0), "tanh": np.tanh,
            "gelu": lambda x: 0.5 * x * (1 + erf(x / np.sqrt(2)))}[act](v)


def _np_dact(act, s):
    from scipy.special import erf

    if act == "relu":
        return (s > 0).astype(np.float64)
    if act == "tanh":
        return 1 - s * s
    return 0.5 * (1 + erf(s / np.sqrt(2))) + s * np.exp(-0.5 * s * s) / np.sqrt(2 * np.pi)


# Shapes the bandwidth-shaped kernels take (K <= 32; N <= 16 with A row-major;
# M <= 16 with B row-major), with leading dimensions padded by `pad` so that
# rows are not 16-byte aligned when pad is odd, and `batch` strided matrices.
SKINNY = [
    # M, N, K, ta, tb, pad, batch, act, dact, beta, preact
    (4096, 1024, 10, 0, 0, 0, 1, "none", "relu", 0.0, False),   # head dgrad with relu'
    (4096, 10, 1024, 0, 1, 0, 1, "relu", None, 0.0, True),      # head forward
    (10, 1024, 4096, 1, 0, 0, 1, "none", None, 1.0, False),     # head wgrad, accumulated
    (2049, 30, 27, 0, 1, 1, 1, "tanh", None, 0.5, False),       # conv1 im2col-like, ragged
    (300, 333, 16, 1, 1, 3, 3, "gelu", None, 0.0, True),        # batched, MN-major A
    (777, 1, 513, 0, 0, 1, 1, "none", "tanh", 0.0, False),      # N = 1, misaligned rows
    (3, 333, 4097, 0, 0, 1, 1, "none", None, 0.0, False),       # M = 3, ragged K
    (16, 96, 8192, 1, 0, 0, 1, "none", "gelu", 0.0, False),     # M = 16, long K
    (8192, 16, 512, 0, 0, 0, 1, "tanh", None, 0.0, False),      # N = 16, B K x N
]


@pytest.mark.parametrize("math", ["fp32", "tf32"])
@pytest.mark.parametrize("case", SKINNY, ids=[f"{c[0]}x{c[1]}x{c[2]}" for c in SKINNY])
def test_skinny_gemm_full_epilogue(tx, math, case):
    """Skinny shapes run exact-fp32 kernels in every math mode: 1e-5 of the
    pre-activation scale even in TF32 mode."""
    from tynx_b200 import _core
    from tynx_b200 import _native as N

    M, Nn, K, ta, tb, pad, batch, act, dact, beta, preact = case
    rng = np.random.default_rng(M + 3 * Nn + 7 * K)
    ar, ac = (K, M) if ta else (M, K)
    br, bc = (Nn, K) if tb else (K, Nn)
    lda, ldb, ldc = ac + pad, bc + pad, Nn + pad
    A = rng.standard_normal((batch, ar, lda)).astype(np.float32)
    B = rng.standard_normal((batch, br, ldb)).astype(np.float32)
    C0 = rng.standard_normal((batch, M, ldc)).astype(np.float32)
    S = rng.standard_normal((batch, M, ldc)).astype(np.float32) * (0.5 if dact == "tanh" else 1)
    bias = rng.standard_normal(Nn).astype(np.float32)
    ctx = _core.context()
    ctx.math = math
    try:
        a, b, c, s, bb = (tx.Tensor(v) for v in (A, B, C0, S, bias))
        p = tx.zeros(batch, M, ldc)
        d = N.GemmDesc()
        d.M, d.N, d.K = M, Nn, K
        d.A, d.lda, d.trans_a = a.ptr, lda, ta
        d.B, d.ldb, d.trans_b = b.ptr, ldb, tb
        d.C, d.ldc = c.ptr, ldc
        d.alpha, d.beta = 0.75, beta
        d.bias, d.bias_scale = bb.ptr, 2.0
        d.act = N.ACT[act]
        if preact:
            d.preact, d.ld_preact = p.ptr, ldc
        if dact:
            d.dact_src, d.ld_dact, d.dact = s.ptr, ldc, N.ACT[dact]
        d.batch = batch
        d.stride_a, d.stride_b, d.stride_c = ar * lda, br * ldb, M * ldc
        ctx.check(N.lib.tx_gemm(ctx.handle, C.byref(d)), "gemm")
        got, got_pre = c.numpy(), p.numpy()
    finally:
        ctx.math = "tf32"
    for z in range(batch):
        Az = A[z, :, :ac].astype(np.float64)
        Bz = B[z, :, :bc].astype(np.float64)
        prod = (Az.T if ta else Az) @ (Bz.T if tb else Bz)
        pre = 0.75 * prod + 2.0 * bias + beta * C0[z, :, :Nn]
        want = _np_act(act, pre)
        if dact:
            want = want * _np_dact(dact, S[z, :, :Nn].astype(np.float64))
        scale = float(np.abs(pre).max())
        assert float(np.abs(got[z, :, :Nn] - want).max()) < 1e-5 * scale
        # padding columns are left alone
        np.testing.assert_array_equal(got[z, :, Nn:], C0[z, :, Nn:])
        if preact:
            assert float(np.abs(got_pre[z, :, :Nn] - pre).max()) < 1e-5 * scale


def _np_round_tf32(x):
    """Round float32 to a 10-bit mantissa, to nearest with ties away from zero
    (add half of the dropped 13-bit field to the magnitude, then truncate)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    sign = u & np.uint32(0x80000000)
    mag = (u & np.uint32(0x7FFFFFFF)) + np.uint32(0x1000)
    return ((mag & np.uint32(0xFFFFE000)) | sign).view(np.float32)


def test_round_tf32_matches_definition(tx):
    from tynx_b200 import _core
    from tynx_b200 import _native as N

    rng = np.random.default_rng(11)
    x = np.concatenate([rng.standard_normal(100003).astype(np.float32) * 1e3,
                        (rng.standard_normal(1000) * 1e-40).astype(np.float32),  # subnormals
                        np.array([0.0, -0.0, 1.0 + 2.0 ** -11, -(1.0 + 2.0 ** -11)], np.float32)])
    ctx = _core.context()
    src = tx.Tensor(x)
    dst = tx.zeros(x.size)
    ctx.check(N.lib.tx_round_tf32(ctx.handle, src.ptr, dst.ptr, x.size))
    np.testing.assert_array_equal(dst.numpy().view(np.uint32), _np_round_tf32(x).view(np.uint32))


@pytest.mark.parametrize("ta,tb", [(0, 1), (1, 0)])
def test_pre_rounded_operands_and_rounded_output(tx, ta, tb):
    """TF32 mode: operands flagged as already rounded skip the kernel's own
    rounding (same bits), and ROUND_OUT stores round_tf32 of the same result."""
    from tynx_b200 import _core
    from tynx_b200 import _native as N

    rng = np.random.default_rng(12)
    M, Nn, K = 1024, 768, 512
    A = _np_round_tf32(rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32))
    B = _np_round_tf32(rng.standard_normal((Nn, K) if tb else (K, Nn)).astype(np.float32))
    bias = rng.standard_normal(Nn).astype(np.float32)
    ctx = _core.context()
    ctx.math = "tf32"
    a, b, bb = tx.Tensor(A), tx.Tensor(B), tx.Tensor(bias)

    def run(flags):
        c = tx.zeros(M, Nn)
        d = N.GemmDesc()
        d.M, d.N, d.K = M, Nn, K
        d.A, d.lda, d.trans_a = a.ptr, A.shape[1], ta
        d.B, d.ldb, d.trans_b = b.ptr, B.shape[1], tb
        d.C, d.ldc = c.ptr, Nn
        d.alpha, d.bias, d.bias_scale, d.act, d.batch = 1.0, bb.ptr, 1.0, N.ACT["relu"], 1
        d.flags = flags
        ctx.check(N.lib.tx_gemm(ctx.handle, C.byref(d)), "gemm")
        return c.numpy()

    base = run(0)
    np.testing.assert_array_equal(run(N.TX_GEMM_A_TF32), base)
    np.testing.assert_array_equal(run(N.TX_GEMM_B_TF32), base)
    np.testing.assert_array_equal(run(N.TX_GEMM_A_TF32 | N.TX_GEMM_B_TF32), base)
    rounded = run(N.TX_GEMM_A_TF32 | N.TX_GEMM_B_TF32 | N.TX_GEMM_ROUND_OUT)
    np.testing.assert_array_equal(rounded.view(np.uint32), _np_round_tf32(base).view(np.uint32))


@pytest.mark.parametrize("M,N,K,ta,tb,dact", [
    (4096, 1024, 1024, 0, 0, "relu"),   # tcgen05 dgrad with act' (TMA epilogue sums)
    (4096, 1024, 10, 0, 0, "relu"),     # small-K head dgrad (block sums)
    (300, 256, 16, 1, 1, "tanh"),       # small-K, MN-major A, ragged rows
    (4096, 10, 1024, 0, 1, None),       # small-N: no fused sums, summed afterwards
    (1000, 384, 200, 0, 1, "gelu"),     # tcgen05 with a ragged last tile
])
@pytest.mark.parametrize("acc", [0, 1])
def test_fused_column_sums(tx, M, N, K, ta, tb, dact, acc):
    """colsum (+)= scale * sum over rows of the unrounded result; C is stored
    either exactly or TF32-rounded (when the kernel fused the sums)."""
    from tynx_b200 import _core
    from tynx_b200 import _native as N_

    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    S = rng.standard_normal((M, N)).astype(np.float32) * 0.5
    prior = rng.standard_normal(N).astype(np.float32)
    ctx = _core.context()
    ctx.math = "tf32"
    a, b, s = tx.Tensor(A), tx.Tensor(B), tx.Tensor(S)

    def run(colsum, flags):
        c = tx.zeros(M, N)
        d = N_.GemmDesc()
        d.M, d.N, d.K = M, N, K
        d.A, d.lda, d.trans_a = a.ptr, A.shape[1], ta
        d.B, d.ldb, d.trans_b = b.ptr, B.shape[1], tb
        d.C, d.ldc = c.ptr, N
        d.alpha, d.batch, d.flags = 1.0, 1, flags
        if dact:
            d.dact_src, d.ld_dact, d.dact = s.ptr, N, N_.ACT[dact]
        if colsum is not None:
            d.colsum, d.colsum_scale, d.colsum_acc = colsum.ptr, 0.5, acc
        ctx.check(N_.lib.tx_gemm(ctx.handle, C.byref(d)), "gemm")
        return c.numpy()

    ref = run(None, 0)
    cs = tx.Tensor(prior)
    got = run(cs, N_.TX_GEMM_ROUND_OUT)
    want = 0.5 * ref.astype(np.float64).sum(axis=0) + (prior if acc else 0)
    scale = float(np.abs(ref).sum(axis=0).max())
    assert float(np.abs(cs.numpy() - want).max()) <= 1e-5 * scale
    assert (got == ref).all() or (got.view(np.uint32) == _np_round_tf32(ref).view(np.uint32)).all()


@pytest.mark.parametrize("tb", [0, 1])
@pytest.mark.parametrize("kind", ["gelu", "gelu_dgrad"])
def test_persistent_gelu_epilogue(tx, kind, tb):
    """More 128 x 256 tiles than SMs and operands already TF32: the persistent
    kernel, whose GELU / GELU' epilogue is shared by eight warps (two per TMEM
    lane quadrant, alternate 32-column chunks).  Against float64 on the same
    operands: C, the stored pre-activation, and the fused column sums of C."""
    from tynx_b200 import _core
    from tynx_b200 import _native as N_

    M, Nn, K = 8192, 1024, 256
    rng = np.random.default_rng(17 + tb)
    A = _np_round_tf32(rng.standard_normal((M, K)).astype(np.float32))
    B = _np_round_tf32((rng.standard_normal((Nn, K) if tb else (K, Nn)) * 0.1).astype(np.float32))
    S = rng.standard_normal((M, Nn)).astype(np.float32)
    bias = rng.standard_normal(Nn).astype(np.float32)
    prior = rng.standard_normal(Nn).astype(np.float32)
    ctx = _core.context()
    ctx.math = "tf32"
    a, b, s, bb, cs = (tx.Tensor(v) for v in (A, B, S, bias, prior))
    c, p = tx.zeros(M, Nn), tx.zeros(M, Nn)
    d = N_.GemmDesc()
    d.M, d.N, d.K = M, Nn, K
    d.A, d.lda, d.trans_a = a.ptr, K, 0
    d.B, d.ldb, d.trans_b = b.ptr, B.shape[1], tb
    d.C, d.ldc = c.ptr, Nn
    d.alpha, d.batch = 0.5, 1
    d.flags = N_.TX_GEMM_A_TF32 | N_.TX_GEMM_B_TF32
    if kind == "gelu":
        d.bias, d.bias_scale, d.act = bb.ptr, 1.0, N_.ACT["gelu"]
        d.preact, d.ld_preact = p.ptr, Nn
    else:
        d.dact_src, d.ld_dact, d.dact = s.ptr, Nn, N_.ACT["gelu"]
        d.colsum, d.colsum_scale, d.colsum_acc = cs.ptr, 0.25, 1
        d.flags |= N_.TX_GEMM_ROUND_OUT
    ctx.check(N_.lib.tx_gemm(ctx.handle, C.byref(d)), "gemm")
    got = c.numpy()
    prod = A.astype(np.float64) @ (B.T if tb else B).astype(np.float64)
    if kind == "gelu":
        pre = 0.5 * prod + bias
        want = _np_act("gelu", pre)
        scale = float(np.abs(pre).max())
        assert float(np.abs(got - want).max()) < 1e-5 * scale
        assert float(np.abs(p.numpy() - pre).max()) < 1e-5 * scale
    else:
        want = 0.5 * prod * _np_dact("gelu", S.astype(np.float64))
        scale = float(np.abs(want).max())
        # C stored TF32-rounded: half a TF32 unit of each value on top
        assert (np.abs(got - want) <= 1e-5 * scale + np.abs(want) * 2.0 ** -11).all()
        np.testing.assert_array_equal(got.view(np.uint32), _np_round_tf32(got).view(np.uint32))
        want_cs = 0.25 * want.sum(axis=0) + prior
        assert float(np.abs(cs.numpy() - want_cs).max()) <= 1e-5 * float(np.abs(want).sum(axis=0).max())


def _strides(shape):
    st, acc = [], 1
    for e in reversed(shape):
        st.append(acc)
        acc *= e
    return st[::-1]


BROADCAST = [
    ((32768, 256), (32768, 256)),            # residual add (one merged axis)
    ((32768, 256), (256,)),                  # bias row
    ((256, 4, 128, 128), ()),                # attention scale
    ((256, 1, 128, 64), (1, 4, 1, 64)),      # both sides broadcast
    ((7, 3, 5), (7, 1, 5)),                  # ragged, not float4-able
    ((4, 6, 1, 2), (6, 3, 1)),
]


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "min", "max", "le", "ge"])
@pytest.mark.parametrize("sa,sb", BROADCAST, ids=[f"{a}-{b}" for a, b in BROADCAST])
def test_broadcast_binary_matches_numpy(tx, op, sa, sb):
    from tynx_b200 import _core
    from tynx_b200 import _native as N

    rng = np.random.default_rng(len(sa) * 7 + len(sb))
    a = rng.standard_normal(sa).astype(np.float32)
    b = (rng.standard_normal(sb) + (3.0 if op == "div" else 0.0)).astype(np.float32)
    shape = np.broadcast_shapes(sa, sb)
    nd = len(shape)

    def bstride(s):
        s = (1,) * (nd - len(s)) + tuple(s)
        st = _strides(s)
        return [0 if s[k] == 1 and shape[k] != 1 else st[k] for k in range(nd)]

    ctx = _core.context()
    A, B, out = tx.Tensor(a), tx.Tensor(b), tx.zeros(*shape)
    ctx.check(N.lib.tx_binary(ctx.handle, N.BIN[op], A.ptr, N.i64_array(bstride(sa)), B.ptr,
                              N.i64_array(bstride(sb)), out.ptr, N.i64_array(shape), nd))
    want = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide,
            "min": np.minimum, "max": np.maximum,
            "le": lambda x, y: (x <= y).astype(np.float32),
            "ge": lambda x, y: (x >= y).astype(np.float32)}[op](a, b)
    np.testing.assert_array_equal(out.numpy(), want.astype(np.float32))


@pytest.mark.parametrize("shape,perm,dtype", [
    ((256, 128, 4, 64), (0, 2, 1, 3), np.float32),   # head split
    ((256, 4, 128, 64), (0, 2, 1, 3), np.float32),   # head merge
    ((512, 3, 33, 17), (0, 2, 3, 1), np.float32),    # NCHW -> NHWC, ragged
    ((256, 128, 4, 64), (0, 2, 3, 1), np.float32),   # attention keys, (s, h*d) -> (h*d, s)
    ((256, 4, 64, 128), (0, 3, 1, 2), np.float32),   # and back (their gradient)
    ((1000, 3), (1, 0), np.float32),
    ((64, 5, 8), (2, 0, 1), np.int64),
])
def test_strided_copy_transposes(tx, shape, perm, dtype):
    from tynx_b200 import _core
    from tynx_b200 import _native as N

    rng = np.random.default_rng(3)
    x = (rng.standard_normal(shape) * 100).astype(dtype)
    st = _strides(shape)
    out_shape = [shape[p] for p in perm]
    ctx = _core.context()
    X = tx.Tensor(x, dtype="int64" if dtype == np.int64 else "float32")
    out = tx.Tensor(np.zeros(out_shape, dtype), dtype="int64" if dtype == np.int64 else "float32")
    ctx.check(N.lib.tx_strided_copy(ctx.handle, X.ptr, N.i64_array([st[p] for p in perm]), out.ptr,
                                    N.i64_array(out_shape), len(shape), x.itemsize))
    np.testing.assert_array_equal(out.numpy(), np.transpose(x, perm))


@pytest.mark.parametrize("shape,keep", [
    ((256, 128, 256), (1, 0, 1)),     # mean over the sequence
    ((512, 128, 8, 8), (1, 1, 0, 0)), # global average pool
    ((32768, 256), (0, 1)),           # bias gradient (column sums)
    ((300, 7, 5), (0, 1, 0)),         # two reduced blocks: generic kernel
    ((8, 9), (1, 1)),                 # nothing reduced
    ((3, 4000), (1, 0)),              # long rows
])
@pytest.mark.parametrize("mean", [0, 1])
def test_reduce_to_matches_numpy(tx, shape, keep, mean):
    from tynx_b200 import _core
    from tynx_b200 import _native as N

    rng = np.random.default_rng(4)
    x = rng.standard_normal(shape).astype(np.float32)
    out_shape = [e if k else 1 for e, k in zip(shape, keep)]
    axes = tuple(i for i, k in enumerate(keep) if not k)
    want = (x.astype(np.float64).mean(axis=axes, keepdims=True) if mean else
            x.astype(np.float64).sum(axis=axes, keepdims=True)) if axes else x.astype(np.float64)
    ctx = _core.context()
    X = tx.Tensor(x)
    prior = rng.standard_normal(out_shape).astype(np.float32)
    for acc in (0, 1):
        out = tx.Tensor(prior)
        ctx.check(N.lib.tx_reduce_to(ctx.handle, X.ptr, N.i64_array(shape), out.ptr,
                                     N.i64_array(out_shape), len(shape), mean, acc))
        expect = want + (prior if acc else 0)
        n_red = int(np.prod([shape[a] for a in axes])) if axes else 1
        tol = 1e-6 * max(1.0, np.sqrt(n_red)) * (1 if mean else np.sqrt(n_red))
        assert np.abs(out.numpy() - expect).max() <= tol * max(1.0, np.abs(x).max()), (acc, n_red)


def test_softmax_xent_matches_oracle(tx):
    from oracle import flex_oracle as fo
    from tynx_b200 import nn

    rng = np.random.default_rng(1)
    for rows, cols in [(4096, 10), (256, 2), (37, 1000), (8192, 16)]:
        z = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
        y = rng.integers(0, cols, rows).astype(np.int64)
        zt = tx.Tensor(z, requires_grad=True)
        loss = nn.functional.cross_entropy(zt, tx.Tensor(y))
        loss.backward()
        ref_z = fo.T(z, requires_grad=True)
        ref = fo.cross_entropy(ref_z, y)
        ref.backward()
        assert abs(loss.item() - ref.item()) <= 1e-5 * max(1.0, abs(ref.item()))
        assert _rel(zt.grad.numpy(), ref_z.grad) < 1e-5


def test_cross_entropy_rejects_out_of_range_labels(tx):
    from tynx_b200 import nn

    z = tx.Tensor(np.zeros((4, 3), np.float32))
    y = tx.Tensor(np.array([0, 1, 3, 2], np.int64))
    with pytest.raises(IndexError):
        nn.functional.cross_entropy(z, y).item()
    # the context stays usable after a latched device error
    assert nn.functional.cross_entropy(z, tx.Tensor(np.array([0, 1, 2, 2], np.int64))).item() == \
        pytest.approx(np.log(3.0), rel=1e-6)


@pytest.mark.parametrize("cols", [256, 100, 1024])  # register-resident rows, scalar path, mixed
def test_layernorm_matches_oracle(tx, cols):
    from oracle import flex_oracle as fo
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    rng = np.random.default_rng(2)
    rows = 3000
    x = rng.standard_normal((rows, cols)).astype(np.float32) * 2 + 1
    g = rng.standard_normal(cols).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    dy = rng.standard_normal((rows, cols)).astype(np.float32)
    X, G, B, DY = (tx.Tensor(v) for v in (x, g, b, dy))
    Y = tx.zeros(rows, cols)
    mean, rstd = tx.zeros(rows), tx.zeros(rows)
    DX, DG, DB = tx.zeros(rows, cols), tx.zeros(cols), tx.zeros(cols)
    ctx.check(N.lib.tx_layernorm_fwd(ctx.handle, X.ptr, G.ptr, B.ptr, Y.ptr, mean.ptr, rstd.ptr,
                                     rows, cols, C.c_float(1e-5)))
    ctx.check(N.lib.tx_layernorm_bwd(ctx.handle, X.ptr, G.ptr, mean.ptr, rstd.ptr, DY.ptr, DX.ptr,
                                     DG.ptr, DB.ptr, rows, cols, 0, 0))
    tx_ = fo.T(x, requires_grad=True)
    tg = fo.T(g, requires_grad=True)
    tb = fo.T(b, requires_grad=True)
    (y,) = fo.layer_norm(tx_, tg, tb, -1, 1e-5, 1)
    y.backward(dy)
    assert _rel(Y.numpy(), y.data) < 1e-5
    assert _rel(DX.numpy(), tx_.grad) < 1e-4
    assert _rel(DG.numpy(), tg.grad) < 1e-4
    assert _rel(DB.numpy(), tb.grad) < 1e-5


@pytest.mark.parametrize("cols", [256, 100])
def test_layernorm_param_grads_accumulate_and_stand_alone(tx, cols):
    """dgamma and dbeta are reduced in one launch when both are wanted; asking
    for one of them, or accumulating into existing values, gives the same
    fixed-order sums bit for bit."""
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    rng = np.random.default_rng(5)
    rows = 2000
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    g = rng.standard_normal(cols).astype(np.float32)
    dy = rng.standard_normal((rows, cols)).astype(np.float32)
    prior_g = rng.standard_normal(cols).astype(np.float32)
    prior_b = rng.standard_normal(cols).astype(np.float32)
    X, G, DY = (tx.Tensor(v) for v in (x, g, dy))
    Y, mean, rstd, DX = tx.zeros(rows, cols), tx.zeros(rows), tx.zeros(rows), tx.zeros(rows, cols)
    ctx.check(N.lib.tx_layernorm_fwd(ctx.handle, X.ptr, G.ptr, tx.zeros(cols).ptr, Y.ptr, mean.ptr,
                                     rstd.ptr, rows, cols, C.c_float(1e-5)))

    def bwd(dg, db, acc):
        ctx.check(N.lib.tx_layernorm_bwd(ctx.handle, X.ptr, G.ptr, mean.ptr, rstd.ptr, DY.ptr, DX.ptr,
                                         dg.ptr if dg is not None else None,
                                         db.ptr if db is not None else None, rows, cols, 0, acc))

    DG, DB = tx.zeros(cols), tx.zeros(cols)
    bwd(DG, DB, 0)
    dg, db = DG.numpy(), DB.numpy()
    only_g, only_b = tx.zeros(cols), tx.zeros(cols)
    bwd(only_g, None, 0)
    bwd(None, only_b, 0)
    np.testing.assert_array_equal(only_g.numpy(), dg)
    np.testing.assert_array_equal(only_b.numpy(), db)
    AG, AB = tx.Tensor(prior_g), tx.Tensor(prior_b)
    bwd(AG, AB, 1)
    np.testing.assert_array_equal(AG.numpy(), prior_g + dg)
    np.testing.assert_array_equal(AB.numpy(), prior_b + db)


def test_adam_is_bit_exact_with_oracle(tx):
    from oracle import flex_oracle as fo
    from tynx_b200 import optim
    from tynx_b200.imported import ImportedModel
    from tynx_b200.workloads import mlp_policy

    wl = mlp_policy()
    model = ImportedModel(wl.onnx)
    params = model.parameters()
    opt = optim.Adam(params, lr=3e-4)
    rng = np.random.default_rng(3)
    ref_params = [fo.T(p.numpy(), requires_grad=True) for p in params]
    ref_opt = fo.Adam(ref_params, lr=3e-4)
    for _ in range(5):
        for p, r in zip(params, ref_params):
            g = rng.standard_normal(p.shape).astype(np.float32)
            p.grad = tx.Tensor(g)
            r.grad = g
        opt.step()
        ref_opt.step()
    for p, r in zip(params, ref_params):
        np.testing.assert_array_equal(p.numpy(), r.data)


def test_adamw_amsgrad_sgd_match_oracle(tx):
    from oracle import flex_oracle as fo
    from tynx_b200 import optim
    from tynx_b200.imported import ImportedModel
    from tynx_b200.workloads import mlp_policy

    rng = np.random.default_rng(4)
    cases = [
        (lambda ps: optim.AdamW(ps, lr=1e-2, weight_decay=0.1),
         lambda ps: fo.Adam(ps, lr=1e-2, weight_decay=0.1, decoupled=True)),
        (lambda ps: optim.Adam(ps, lr=1e-2, amsgrad=True, weight_decay=0.01),
         lambda ps: fo.Adam(ps, lr=1e-2, amsgrad=True, weight_decay=0.01)),
        (lambda ps: optim.SGD(ps, lr=0.1, momentum=0.9, nesterov=True),
         lambda ps: fo.SGD(ps, lr=0.1, momentum=0.9, nesterov=True)),
        (lambda ps: optim.SGD(ps, lr=0.1, momentum=0.5, dampening=0.1, weight_decay=0.01),
         lambda ps: fo.SGD(ps, lr=0.1, momentum=0.5, dampening=0.1, weight_decay=0.01)),
    ]
    for make, make_ref in cases:
        model = ImportedModel(mlp_policy().onnx)
        params = model.parameters()
        opt = make(params)
        refs = [fo.T(p.numpy(), requires_grad=True) for p in params]
        ref_opt = make_ref(refs)
        for _ in range(4):
            for p, r in zip(params, refs):
                g = rng.standard_normal(p.shape).astype(np.float32)
                p.grad = tx.Tensor(g)
                r.grad = g
            opt.step()
            ref_opt.step()
        for p, r in zip(params, refs):
            np.testing.assert_allclose(p.numpy(), r.data, rtol=1e-6, atol=1e-7)


def test_gather_scatter_rows(tx):
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    rng = np.random.default_rng(6)
    table = rng.standard_normal((1000, 256)).astype(np.float32)
    idx = rng.integers(-1000, 1000, 5000).astype(np.int64)
    T, I = tx.Tensor(table), tx.Tensor(idx)
    out = tx.zeros(5000, 256)
    ctx.check(N.lib.tx_gather_rows(ctx.handle, T.ptr, 1000, 256, I.ptr, 5000, out.ptr))
    np.testing.assert_array_equal(out.numpy(), table[np.where(idx < 0, idx + 1000, idx)])
    src = rng.integers(-3, 4, (5000, 256)).astype(np.float32)  # integers: exact in any order
    acc = tx.zeros(1000, 256)
    ctx.check(N.lib.tx_scatter_add_rows(ctx.handle, acc.ptr, 1000, 256, I.ptr, 5000,
                                        tx.Tensor(src).ptr))
    want = np.zeros((1000, 256), np.float32)
    np.add.at(want, np.where(idx < 0, idx + 1000, idx), src)
    np.testing.assert_array_equal(acc.numpy(), want)


def test_bias_grad_and_reductions(tx):
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    rng = np.random.default_rng(8)
    for M, Nn in [(4096, 1024), (8192, 16), (7, 3), (32768, 256)]:
        dy = rng.standard_normal((M, Nn)).astype(np.float32)
        db = tx.zeros(Nn)
        ctx.check(N.lib.tx_bias_grad(ctx.handle, tx.Tensor(dy).ptr, db.ptr, M, Nn, C.c_float(1.0), 0))
        assert _rel(db.numpy(), dy.astype(np.float64).sum(0)) < 1e-5
    x = rng.standard_normal((16, 33, 8)).astype(np.float32)
    t = tx.Tensor(x)
    np.testing.assert_allclose(t.mean(1).numpy(), x.mean(1), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(t.sum().numpy(), [x.astype(np.float64).sum()], rtol=1e-5)


def test_gelu_and_derivative_within_2e7_of_float64(tx):
    """GELU and GELU' of the elementwise kernels (the GEMM epilogues share the
    same device functions) against float64 erf over [-12, 12] and a few edge
    values: absolute error at most 3e-7 * max(1, |x|)."""
    from scipy.special import erf

    x = np.concatenate([np.linspace(-12.0, 12.0, 240001),
                        [0.0, -0.0, 1e-30, -1e-30, 1e-6, -1e-6, 0.75, -0.75]]).astype(np.float32)
    t = tx.Tensor(x, requires_grad=True)
    y = t.gelu()
    y.sum().backward()
    x64 = x.astype(np.float64)
    cdf = 0.5 * (1.0 + erf(x64 / np.sqrt(2.0)))
    pdf = np.exp(-0.5 * x64 * x64) / np.sqrt(2.0 * np.pi)
    bound = 3e-7 * np.maximum(1.0, np.abs(x64))
    err_y = np.abs(y.numpy().astype(np.float64) - x64 * cdf)
    err_g = np.abs(t.grad.numpy().astype(np.float64) - (cdf + x64 * pdf))
    assert np.all(err_y <= bound), float((err_y / bound).max())
    assert np.all(err_g <= bound), float((err_g / bound).max())


def _tf32_rn(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


@pytest.mark.parametrize("math,split,tol", [("tf32", False, 2e-3), ("3xtf32", False, 1e-5), ("fp32", False, 1e-5),
                                            ("tf32", True, 5e-5)])
@pytest.mark.parametrize("M,N,K", [(4096, 256, 256), (32768, 256, 256), (300, 96, 64)])
def test_batched_product_with_shared_a(tx, math, split, tol, M, N, K):
    """TX_GEMM_A_SHARED: one A for a batch of three B stored back to back
    (with padding between them) into three C slices, equal to the three
    products.  split: the engine's form for projections, the weights as a
    TF32 head and tail (B_lo) and A already TF32, compared with A_tf32 @ B."""
    import ctypes as C

    from tynx_b200 import _core
    from tynx_b200 import _native as N_

    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    spacing = K * N + 64
    Bflat = rng.standard_normal(3 * spacing).astype(np.float32)
    Bs = [Bflat[z * spacing:z * spacing + K * N].reshape(K, N) for z in range(3)]
    ctx = _core.context()
    ctx.math = math
    try:
        flags = N_.TX_GEMM_A_SHARED
        if split:
            A = _tf32_rn(A)
            head = _tf32_rn(Bflat)
            tail = _tf32_rn(Bflat - head)
            b, blo = tx.Tensor(head), tx.Tensor(tail)
            flags |= N_.TX_GEMM_A_TF32 | N_.TX_GEMM_B_TF32
        else:
            b, blo = tx.Tensor(Bflat), None
        a = tx.Tensor(A)
        c = tx.Tensor(np.zeros((3, M, N), np.float32))
        d = N_.GemmDesc()
        d.M, d.N, d.K = M, N, K
        d.A, d.lda, d.trans_a = a.ptr, K, 0
        d.B, d.ldb, d.trans_b = b.ptr, N, 0
        d.C, d.ldc = c.ptr, N
        d.alpha, d.bias_scale = 1.0, 1.0
        d.batch, d.stride_a, d.stride_b, d.stride_c = 3, 0, spacing, M * N
        d.flags = flags
        if blo is not None:
            d.B_lo = blo.ptr
        ctx.check(N_.lib.tx_gemm(ctx.handle, C.byref(d)), "gemm")
        got = c.numpy()
    finally:
        ctx.math = "tf32"
    A64 = A.astype(np.float64)
    for z in range(3):
        ref = A64 @ Bs[z].astype(np.float64)
        err = np.linalg.norm(got[z] - ref) / np.linalg.norm(ref)
        assert err <= tol, (z, err)
