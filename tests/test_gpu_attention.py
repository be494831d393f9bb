"""Fused tcgen05 attention (``tx_attention_fwd`` / ``tx_attention_bwd``).

Against a float64 numpy restatement of the unfused block the reference runs
(MatMul(Q, K^T) * scale -> Softmax -> MatMul(., V) per head over the merged
[batch * seq, heads * 64] layout, and its gradients): the TF32 products
(operands rounded to nearest, 10-bit mantissas) are held to 2e-3 of each
output's scale; masked positions (sequences shorter than the 128-row tile)
contribute nothing; the three gradients accumulate into existing values on
request.  Through the engine, the transformer workload's fused step is checked
against the oracle by test_gpu_parity.py; here a sequence length that leaves
most of the tile masked runs through ``tx.load`` too.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref(q, k, v, dout, B, S, H, scale):
    D = 64
    q4 = q.astype(np.float64).reshape(B, S, H, D).transpose(0, 2, 1, 3)
    k4 = k.astype(np.float64).reshape(B, S, H, D).transpose(0, 2, 1, 3)
    v4 = v.astype(np.float64).reshape(B, S, H, D).transpose(0, 2, 1, 3)
    s = q4 @ k4.transpose(0, 1, 3, 2) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = p @ v4
    do4 = dout.astype(np.float64).reshape(B, S, H, D).transpose(0, 2, 1, 3)
    dp = do4 @ v4.transpose(0, 1, 3, 2)
    ds = p * (dp - (p * dp).sum(-1, keepdims=True)) * scale
    dq = ds @ k4
    dk = ds.transpose(0, 1, 3, 2) @ q4
    dv = p.transpose(0, 1, 3, 2) @ do4
    merge = lambda t: t.transpose(0, 2, 1, 3).reshape(B * S, H * D)  # noqa: E731
    return merge(o), merge(dq), merge(dk), merge(dv)


def _scaled_err(a, b):
    return float(np.abs(a - b).max()) / max(float(np.abs(b).max()), 1e-30)


@pytest.mark.parametrize("B,S,H", [(3, 128, 4), (5, 77, 2), (2, 1, 1), (4, 100, 3)])
@pytest.mark.parametrize("acc", [0, 1])
def test_fused_attention_matches_fp64(B, S, H, acc):
    import tynx_b200 as tx
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    rng = np.random.default_rng(B * 100 + S + H)
    E = H * 64
    q, k, v, dout = (rng.standard_normal((B * S, E)).astype(np.float32) for _ in range(4))
    scale = 0.125
    Q, K, V, DO = (tx.Tensor(a) for a in (q, k, v, dout))
    O = tx.zeros(B * S, E)
    base = [rng.standard_normal((B * S, E)).astype(np.float32) if acc else np.zeros((B * S, E), np.float32)
            for _ in range(3)]
    DQ, DK, DV = (tx.Tensor(a) for a in base)
    ctx.check(N.lib.tx_attention_fwd(ctx.handle, Q.ptr, K.ptr, V.ptr, E, O.ptr, E, B, S, H, 64,
                                     C.c_float(scale), 0))
    ctx.check(N.lib.tx_attention_bwd(ctx.handle, Q.ptr, K.ptr, V.ptr, E, DO.ptr, E, DQ.ptr, DK.ptr, DV.ptr,
                                     E, B, S, H, 64, C.c_float(scale), 2 if acc else 0))
    o, dq, dk, dv = _ref(q, k, v, dout, B, S, H, scale)
    assert _scaled_err(O.numpy(), o) < 2e-3
    for got, want, b0 in ((DQ, dq, base[0]), (DK, dk, base[1]), (DV, dv, base[2])):
        assert _scaled_err(got.numpy() - b0, want) < 2e-3


def test_fused_attention_rejects_unsupported_shapes():
    import tynx_b200 as tx
    from tynx_b200 import _native as N
    from tynx_b200._core import context

    ctx = context()
    a = tx.zeros(256, 256)
    with pytest.raises(Exception, match="sequence length"):
        ctx.check(N.lib.tx_attention_fwd(ctx.handle, a.ptr, a.ptr, a.ptr, 256, a.ptr, 256, 1, 256, 4, 64,
                                         C.c_float(1.0), 0))
    with pytest.raises(Exception, match="head dimension"):
        ctx.check(N.lib.tx_attention_fwd(ctx.handle, a.ptr, a.ptr, a.ptr, 256, a.ptr, 256, 2, 128, 8, 32,
                                         C.c_float(1.0), 0))


def test_short_sequence_transformer_step_matches_oracle():
    """A transformer whose sequences (77) fill part of the attention tile: one
    TF32 training step through the fused path against the float64 oracle."""
    import tynx_b200 as tx
    from oracle import flex_oracle as fo
    from tynx_b200 import workloads
    from tynx_b200.onnx import ir

    tx.set_math_mode("tf32")
    wl = workloads.transformer(batch=8, seq=77)
    model = tx.load(wl.onnx, trainable="auto")
    b = wl.make_batch(0)
    loss = tx.nn.functional.cross_entropy(model(tx.Tensor(b["ids"], dtype="int64")), tx.Tensor(b["y"]))
    loss.backward()
    with fo.precision(np.float64):
        ref = fo.OracleModel(ir.load_training_graph(wl.onnx))
        rl = fo.cross_entropy(ref(b["ids"]), b["y"])
        rl.backward()
    assert abs(loss.item() - rl.item()) <= 1e-3 * max(1.0, abs(rl.item()))
    params = dict(model.named_parameters())
    for n, p in ref.named_parameters():
        g = params[n].grad.numpy().astype(np.float64)
        err = np.linalg.norm(g - p.grad) / np.linalg.norm(p.grad)
        assert err < 3e-3, (n, err)
