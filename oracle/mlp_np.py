"""numpy restatement of the MLP training-step oracle, for the BASELINE-sized configs.

TEST INFRASTRUCTURE ONLY (the checker): imported by tests/ alone, never by the
product path.

It computes exactly what ``orc_mlp_train`` in oracle.cpp computes (the
multi-layer extension of pkt's ``cpu_train_linear``, examples/train_linear.cu:101-151,
with pkt's MSE scaling from include/ops/mse.cuh:36-60 and SGD from
include/ops/sgd.cuh:33-44): the same bf16 storage / TF32 operand rounding, float
bias add and ReLU, fp64 accumulation of every GEMM. The GEMMs go through numpy's
float64 matmul (products of float32 operands are exact in float64; only the order
of the fp64 sums differs from oracle.cpp's loops), so one step of the 4-layer
4096-wide configuration takes seconds instead of the C loops' tens of seconds.
``tests/test_oracle.py`` checks the two restatements against each other.
"""
import numpy as np


def bf16_round(a):
    """Round-to-nearest-even to bfloat16, returned as float32 (NaN kept quiet)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + np.uint32(0x7FFF) + ((u >> 16) & 1)) & np.uint32(0xFFFF0000)
    if nan.any():
        r = np.where(nan, (u | 0x00400000) & 0xFFFF0000, r).astype(np.uint32)
    return r.view(np.float32)


def tf32_round(a):
    """TF32 operand as the TMA unit produces it from fp32: nearest even at 10
    mantissa bits; Inf / NaN passed through."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    special = (u & 0x7F800000) == 0x7F800000
    r = (u + np.uint32(0xFFF) + ((u >> 13) & 1)) & np.uint32(0xFFFFE000)
    r = np.where(special, u, r).astype(np.uint32)
    return r.view(np.float32)


def _store(mode, a):
    return bf16_round(a) if mode == "bf16" else np.asarray(a, np.float32)


def _operand(mode, a):
    if mode == "bf16":
        return bf16_round(a)
    if mode == "tf32":
        return tf32_round(a)
    return np.asarray(a, np.float32)


def _mm(a, b):
    """fp64 product of float32 operands, rounded once to float32."""
    return np.matmul(a.astype(np.float64), b.astype(np.float64)).astype(np.float32)


def _mm32(a, b):
    """The same product accumulated in float32 (numpy's sgemm)."""
    return np.matmul(np.asarray(a, np.float32), np.asarray(b, np.float32))


def mlp_train(dims, x, t, Ws, bs, lr, steps, mode="bf16", want_grads=False, relu_last=False,
              accum="fp64"):
    """Same contract as oracle.mlp_train (oracle.cpp orc_mlp_train).

    accum="fp32" evaluates the same rounded arithmetic with float32 GEMM
    accumulation, as any fp32-accumulating implementation does (the GPU's tensor
    cores among them); the distance between the two evaluations is the
    conditioning floor of a comparison against the fp64 truth.

    Returns dict(W, b, losses[, dW, db]) with the gradients of the last step."""
    mm = _mm if accum == "fp64" else _mm32
    L = len(dims) - 1
    B = x.shape[0]
    W = [np.array(w, np.float32, copy=True) for w in Ws]
    b = None if bs is None else [np.array(v, np.float32, copy=True) for v in bs]
    H0 = _store(mode, x)
    tq = _store(mode, t)
    dout = dims[L]
    inv = 1.0 / (float(B) * float(dout))
    scale = np.float32(2.0 * inv)
    losses = np.zeros(steps, np.float32)
    dW = db = None
    for step in range(steps):
        Wop = [_operand(mode, w) for w in W]
        H = [H0]
        for l in range(L):
            p = mm(_operand(mode, H[l]), Wop[l].T)
            if b is not None:
                p = p + b[l][None, :]
            if l < L - 1 or relu_last:
                p = np.maximum(p, np.float32(0))
            H.append(p if l == L - 1 else _store(mode, p))
        Y = H[L]
        diff = Y - tq
        d64 = diff.astype(np.float64)
        losses[step] = np.float32(np.sum(d64 * d64) * inv)
        g = scale * diff
        if relu_last:
            g = np.where(Y <= 0, np.float32(0), g)
        dY = _store(mode, g)
        dW = [None] * L
        db = [None] * L
        for l in range(L - 1, -1, -1):
            dYop = _operand(mode, dY)
            dW[l] = mm(dYop.T, _operand(mode, H[l]))
            if b is not None:
                db[l] = np.sum(dY.astype(np.float64), axis=0).astype(np.float32)
            if l > 0:
                v = mm(dYop, Wop[l])
                v = np.where(H[l] > 0, v, np.float32(0))
                dY = _store(mode, v)
        nlr = np.float64(np.float32(-lr))
        for l in range(L):
            W[l] = (nlr * dW[l].astype(np.float64) + W[l].astype(np.float64)).astype(np.float32)
            if b is not None:
                b[l] = (nlr * db[l].astype(np.float64) + b[l].astype(np.float64)).astype(np.float32)
    out = {"W": W, "b": b, "losses": losses}
    if want_grads:
        out["dW"] = dW
        out["db"] = db
    return out
