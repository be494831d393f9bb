"""The five training workloads: seeded ONNX models and synthetic input streams.

The reference builds its benchmark models with a small protobuf writer
(``benchmarks/crates/protocol/src/training.rs:303-336``); the same is done here
with :mod:`tynx_b200.onnx.proto`.  Weights are drawn from numpy PCG64 with the
formulas of ``crates/tynx-python/python/tynx/nn/init.py:79-105``
(Xavier-uniform bound sqrt(6/(fan_in+fan_out)), Kaiming-uniform bound
sqrt(6/fan_in)); biases are zero.  Batches come from PCG64 seeded with
``base_seed + step`` so that every implementation sees identical data.

Weights follow the PyTorch export convention: ``Gemm(x, W[out,in], b, transB=1)``.

Workloads
  mlp_policy      64->256 tanh ->256 tanh ->8, batch 256, Adam 3e-4
  mlp_classifier  784->1024 relu ->1024 relu ->10, batch 4096, Adam 1e-3
  ppo             trunk 128->512 tanh ->512 tanh; policy head 512->16, value head 512->1;
                  minibatch 8192 of a 65536 rollout; Adam 3e-4
  cnn             conv3x3 3->32 p1, conv3x3 32->64 s2 p1, conv3x3 64->128 s2 p1 (relu),
                  global average pool, Gemm 128->10; batch 512; Adam 1e-3
  transformer     token + learned positional embedding (8192x256, 128x256), 4 pre-norm
                  layers (d 256, 4 heads, FFN 1024 GELU), mean-pool, Gemm 256->2;
                  batch 256 x 128 tokens; Adam 1e-4
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from .onnx import proto

F32 = np.float32


def xavier(rng, fan_out: int, fan_in: int, shape=None) -> np.ndarray:
    bound = math.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-bound, bound, size=shape or (fan_out, fan_in)).astype(F32)


def kaiming(rng, fan_out: int, fan_in: int, shape=None) -> np.ndarray:
    bound = math.sqrt(6.0 / fan_in)
    return rng.uniform(-bound, bound, size=shape or (fan_out, fan_in)).astype(F32)


@dataclass
class Workload:
    name: str
    onnx: bytes
    batch: int
    lr: float
    loss: str  # "cross_entropy" | "ppo"
    make_batch: Callable[[int], dict]
    dense_weights: int  # sum of weight-matrix elements (FLOP convention 6*B*sum)
    params: int
    flop_per_step: float
    notes: dict = field(default_factory=dict)


def _gemm_chain(dims, act, init, seed, *, opset=13, name="mlp"):
    rng = np.random.default_rng(seed)
    nodes, inits = [], []
    prev = "x"
    for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
        w = init(rng, dout, din)
        inits.append(proto.encode_tensor(f"fc{i}.weight", w))
        inits.append(proto.encode_tensor(f"fc{i}.bias", np.zeros(dout, F32)))
        out = "logits" if i == len(dims) - 2 else f"h{i}_pre"
        nodes.append(proto.encode_node("Gemm", [prev, f"fc{i}.weight", f"fc{i}.bias"], [out],
                                       name=f"fc{i}", transB=1))
        if i < len(dims) - 2:
            nodes.append(proto.encode_node(act, [out], [f"h{i}"], name=f"act{i}"))
            prev = f"h{i}"
    model = proto.encode_model(
        nodes, inits, [proto.encode_value_info("x", proto.FLOAT, ["batch", dims[0]])],
        [proto.encode_value_info("logits", proto.FLOAT, ["batch", dims[-1]])],
        graph_name=name, opset=opset)
    weights = sum(a * b for a, b in zip(dims[:-1], dims[1:]))
    return model, weights, weights + sum(dims[1:])


def mlp_policy(batch: int = 256, seed: int = 0) -> Workload:
    dims = [64, 256, 256, 8]
    model, w, p = _gemm_chain(dims, "Tanh", xavier, seed, name="mlp_policy")

    def make(step: int) -> dict:
        rng = np.random.default_rng(1000 + step)
        return {"x": rng.standard_normal((batch, 64)).astype(F32),
                "y": rng.integers(0, 8, size=batch, dtype=np.int64)}

    return Workload("mlp_policy", model, batch, 3e-4, "cross_entropy", make, w, p, 6.0 * batch * w)


def mlp_classifier(batch: int = 4096, seed: int = 0) -> Workload:
    dims = [784, 1024, 1024, 10]
    model, w, p = _gemm_chain(dims, "Relu", kaiming, seed, name="mlp_classifier")

    def make(step: int) -> dict:
        rng = np.random.default_rng(1000 + step)
        return {"x": rng.random((batch, 784), dtype=F32),
                "y": rng.integers(0, 10, size=batch, dtype=np.int64)}

    return Workload("mlp_classifier", model, batch, 1e-3, "cross_entropy", make, w, p,
                    6.0 * batch * w)


def ppo(minibatch: int = 8192, rollout: int = 65536, seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    nodes, inits = [], []
    shapes = [(128, 512), (512, 512)]
    prev = "obs"
    for i, (din, dout) in enumerate(shapes):
        inits += [proto.encode_tensor(f"trunk{i}.weight", xavier(rng, dout, din)),
                  proto.encode_tensor(f"trunk{i}.bias", np.zeros(dout, F32))]
        nodes += [proto.encode_node("Gemm", [prev, f"trunk{i}.weight", f"trunk{i}.bias"],
                                    [f"t{i}_pre"], name=f"trunk{i}", transB=1),
                  proto.encode_node("Tanh", [f"t{i}_pre"], [f"t{i}"], name=f"tanh{i}")]
        prev = f"t{i}"
    for head, n in (("policy", 16), ("value", 1)):
        inits += [proto.encode_tensor(f"{head}.weight", xavier(rng, n, 512)),
                  proto.encode_tensor(f"{head}.bias", np.zeros(n, F32))]
        out = "logits" if head == "policy" else "value"
        nodes.append(proto.encode_node("Gemm", [prev, f"{head}.weight", f"{head}.bias"], [out],
                                       name=head, transB=1))
    model = proto.encode_model(
        nodes, inits, [proto.encode_value_info("obs", proto.FLOAT, ["batch", 128])],
        [proto.encode_value_info("logits", proto.FLOAT, ["batch", 16]),
         proto.encode_value_info("value", proto.FLOAT, ["batch", 1])],
        graph_name="ppo_actor_critic", opset=13)
    w = 128 * 512 + 512 * 512 + 512 * 16 + 512
    params = w + 512 + 512 + 16 + 1

    data_rng = np.random.default_rng(7)
    rollout_obs = data_rng.standard_normal((rollout, 128)).astype(F32)
    rollout_actions = data_rng.integers(0, 16, size=rollout, dtype=np.int64)
    rollout_adv = data_rng.standard_normal(rollout).astype(F32)
    rollout_ret = data_rng.standard_normal(rollout).astype(F32)

    def make(step: int) -> dict:
        per_epoch = rollout // minibatch
        order = np.random.default_rng(2000 + step // per_epoch).permutation(rollout)
        idx = order[(step % per_epoch) * minibatch:(step % per_epoch + 1) * minibatch]
        return {"obs": rollout_obs[idx], "actions": rollout_actions[idx],
                "advantages": rollout_adv[idx], "returns": rollout_ret[idx], "index": idx}

    wl = Workload("ppo", model, minibatch, 3e-4, "ppo", make, w, params, 6.0 * minibatch * w)
    wl.notes = {"rollout": rollout, "rollout_obs": rollout_obs}
    return wl


def cnn(batch: int = 512, seed: int = 0) -> Workload:
    """Conv padding: BASELINE names none for the stride-2 convs; pad 1 is fixed here
    (32x32 -> 32x32 -> 16x16 -> 8x8)."""
    rng = np.random.default_rng(seed)
    nodes, inits = [], []
    chans = [(3, 32, 1), (32, 64, 2), (64, 128, 2)]
    prev = "x"
    for i, (cin, cout, stride) in enumerate(chans):
        w = kaiming(rng, cout, cin * 9, shape=(cout, cin, 3, 3))
        inits += [proto.encode_tensor(f"conv{i}.weight", w),
                  proto.encode_tensor(f"conv{i}.bias", np.zeros(cout, F32))]
        nodes += [proto.encode_node("Conv", [prev, f"conv{i}.weight", f"conv{i}.bias"],
                                    [f"c{i}"], name=f"conv{i}", kernel_shape=[3, 3],
                                    pads=[1, 1, 1, 1], strides=[stride, stride]),
                  proto.encode_node("Relu", [f"c{i}"], [f"r{i}"], name=f"relu{i}")]
        prev = f"r{i}"
    nodes.append(proto.encode_node("GlobalAveragePool", [prev], ["pooled"], name="gap"))
    nodes.append(proto.encode_node("Flatten", ["pooled"], ["features"], name="flatten", axis=1))
    inits += [proto.encode_tensor("head.weight", kaiming(rng, 10, 128)),
              proto.encode_tensor("head.bias", np.zeros(10, F32))]
    nodes.append(proto.encode_node("Gemm", ["features", "head.weight", "head.bias"], ["logits"],
                                   name="head", transB=1))
    model = proto.encode_model(
        nodes, inits, [proto.encode_value_info("x", proto.FLOAT, ["batch", 3, 32, 32])],
        [proto.encode_value_info("logits", proto.FLOAT, ["batch", 10])],
        graph_name="small_cnn", opset=13)
    params = 32 * 27 + 32 + 64 * 288 + 64 + 128 * 576 + 128 + 1280 + 10
    macs = 32 * 32 * 32 * 27 + 64 * 16 * 16 * 288 + 128 * 8 * 8 * 576 + 1280

    def make(step: int) -> dict:
        r = np.random.default_rng(1000 + step)
        return {"x": r.standard_normal((batch, 3, 32, 32)).astype(F32),
                "y": r.integers(0, 10, size=batch, dtype=np.int64)}

    return Workload("cnn", model, batch, 1e-3, "cross_entropy", make, params - 234, params,
                    6.0 * batch * macs, notes={"padding": 1})


def transformer(batch: int = 256, seq: int = 128, vocab: int = 8192, d: int = 256,
                heads: int = 4, layers: int = 4, ffn: int = 1024, seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    hd = d // heads
    nodes, inits = [], []

    def const(name, array):
        nodes.append(proto.encode_node("Constant", [], [name], name=name + "_const",
                                       value=np.asarray(array)))

    inits.append(proto.encode_tensor("tok_emb.weight", (rng.standard_normal((vocab, d)) * 0.02).astype(F32)))
    inits.append(proto.encode_tensor("pos_emb.weight", (rng.standard_normal((seq, d)) * 0.02).astype(F32)))
    inits.append(proto.encode_tensor("pos_ids", np.arange(seq, dtype=np.int64)))
    nodes.append(proto.encode_node("Gather", ["tok_emb.weight", "ids"], ["tok"], name="tok_emb", axis=0))
    nodes.append(proto.encode_node("Gather", ["pos_emb.weight", "pos_ids"], ["pos"], name="pos_emb", axis=0))
    nodes.append(proto.encode_node("Add", ["tok", "pos"], ["x0"], name="embed_add"))
    const("split_shape", np.asarray([0, 0, heads, hd], np.int64))
    const("merge_shape", np.asarray([0, 0, d], np.int64))
    const("attn_scale", np.asarray(1.0 / math.sqrt(hd), np.float32))
    x = "x0"
    for l in range(layers):
        p = f"layer{l}"
        for ln in ("ln1", "ln2"):
            inits += [proto.encode_tensor(f"{p}.{ln}.weight", np.ones(d, F32)),
                      proto.encode_tensor(f"{p}.{ln}.bias", np.zeros(d, F32))]
        for proj in ("q", "k", "v", "o"):
            inits.append(proto.encode_tensor(f"{p}.{proj}.weight", xavier(rng, d, d, shape=(d, d))))
        inits.append(proto.encode_tensor(f"{p}.ffn1.weight", xavier(rng, ffn, d, shape=(d, ffn))))
        inits.append(proto.encode_tensor(f"{p}.ffn2.weight", xavier(rng, d, ffn, shape=(ffn, d))))
        n = lambda *a, **k: nodes.append(proto.encode_node(*a, **k))  # noqa: E731
        n("LayerNormalization", [x, f"{p}.ln1.weight", f"{p}.ln1.bias"], [f"{p}.h1"], name=f"{p}.ln1",
          axis=-1, epsilon=1e-5)
        for proj in ("q", "k", "v"):
            n("MatMul", [f"{p}.h1", f"{p}.{proj}.weight"], [f"{p}.{proj}"], name=f"{p}.{proj}_proj")
            n("Reshape", [f"{p}.{proj}", "split_shape"], [f"{p}.{proj}s"], name=f"{p}.{proj}_split")
        n("Transpose", [f"{p}.qs"], [f"{p}.qh"], name=f"{p}.q_t", perm=[0, 2, 1, 3])
        n("Transpose", [f"{p}.ks"], [f"{p}.kh"], name=f"{p}.k_t", perm=[0, 2, 3, 1])
        n("Transpose", [f"{p}.vs"], [f"{p}.vh"], name=f"{p}.v_t", perm=[0, 2, 1, 3])
        n("MatMul", [f"{p}.qh", f"{p}.kh"], [f"{p}.scores"], name=f"{p}.qk")
        n("Mul", [f"{p}.scores", "attn_scale"], [f"{p}.scaled"], name=f"{p}.scale")
        n("Softmax", [f"{p}.scaled"], [f"{p}.probs"], name=f"{p}.softmax", axis=-1)
        n("MatMul", [f"{p}.probs", f"{p}.vh"], [f"{p}.ctx"], name=f"{p}.pv")
        n("Transpose", [f"{p}.ctx"], [f"{p}.ctx_t"], name=f"{p}.ctx_t", perm=[0, 2, 1, 3])
        n("Reshape", [f"{p}.ctx_t", "merge_shape"], [f"{p}.merged"], name=f"{p}.merge")
        n("MatMul", [f"{p}.merged", f"{p}.o.weight"], [f"{p}.attn"], name=f"{p}.o_proj")
        n("Add", [x, f"{p}.attn"], [f"{p}.r1"], name=f"{p}.res1")
        n("LayerNormalization", [f"{p}.r1", f"{p}.ln2.weight", f"{p}.ln2.bias"], [f"{p}.h2"],
          name=f"{p}.ln2", axis=-1, epsilon=1e-5)
        n("MatMul", [f"{p}.h2", f"{p}.ffn1.weight"], [f"{p}.f1"], name=f"{p}.ffn1")
        n("Gelu", [f"{p}.f1"], [f"{p}.g"], name=f"{p}.gelu")
        n("MatMul", [f"{p}.g", f"{p}.ffn2.weight"], [f"{p}.f2"], name=f"{p}.ffn2")
        n("Add", [f"{p}.r1", f"{p}.f2"], [f"{p}.out"], name=f"{p}.res2")
        x = f"{p}.out"
    nodes.append(proto.encode_node("ReduceMean", [x], ["pooled"], name="mean_pool", axes=[1],
                                   keepdims=0))
    inits += [proto.encode_tensor("head.weight", xavier(rng, 2, d)),
              proto.encode_tensor("head.bias", np.zeros(2, F32))]
    nodes.append(proto.encode_node("Gemm", ["pooled", "head.weight", "head.bias"], ["logits"],
                                   name="head", transB=1))
    model = proto.encode_model(
        nodes, inits, [proto.encode_value_info("ids", proto.INT64, ["batch", seq])],
        [proto.encode_value_info("logits", proto.FLOAT, ["batch", 2])],
        graph_name="transformer_encoder", opset=20)
    dense = layers * (4 * d * d + 2 * d * ffn)
    params = vocab * d + seq * d + dense + layers * 4 * d + 2 * d + 2
    tokens = batch * seq
    attn = 3 * layers * (4 * batch * heads * seq * seq * hd)
    flop = 6.0 * tokens * dense + attn

    def make(step: int) -> dict:
        r = np.random.default_rng(1000 + step)
        return {"ids": r.integers(0, vocab, size=(batch, seq), dtype=np.int64),
                "y": r.integers(0, 2, size=batch, dtype=np.int64)}

    return Workload("transformer", model, batch, 1e-4, "cross_entropy", make, dense, params, flop)


WORKLOADS = {
    "mlp_policy": mlp_policy,
    "mlp_classifier": mlp_classifier,
    "ppo": ppo,
    "cnn": cnn,
    "transformer": transformer,
}
