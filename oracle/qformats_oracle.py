"""CPU oracle for the q8_0 / q4_0 GEMV path (test infrastructure only).

This module is the checker, never the product: only the tests, the smoke
check and the CPU-baseline leg of the benchmark import it.  Nothing in
``qgemv_roofline_b200`` may call it.

It restates, in numpy, the reference's algorithm for the path:

* ``quantize_q8_0``   follows python/qformats.py:17-25 (and its C++ twin
  src/bench.cu:32-47): per 32-weight block ``amax = max|w|``,
  ``d = amax / 127`` (fp32, correctly rounded), ``id = 1/d`` when ``d > 0``
  else 0, ``q = clamp(round_half_even(w * id), -127, 127)``, ``d`` stored as
  fp16 (round to nearest even).
* ``quantize_q4_0``   follows python/qformats.py:28-40 (twin bench.cu:49-69):
  ``mx`` = signed value at the first index of the largest ``|w|``,
  ``d = mx / -8``, ``id = 1/d`` when ``d != 0`` else 0,
  ``q = clamp(trunc(fp32(fp32(w * id) + 8.5)), 0, 15)`` (two roundings, no
  fused multiply-add), packed byte ``i`` of a block = ``q[i] | q[i+16] << 4``.
* ``dequant_q8_0`` / ``dequant_q4_0`` follow python/qformats.py:43-56
  (``dequant_torch`` restates them in torch on the CPU, the reference's own
  CPU GEMV path, for the timed CPU baseline only).
* ``matvec_ref``      is the float64 dequant-matvec of src/bench.cu:75-111,
  the ground truth every kernel is checked against.
* ``check_rowwise`` / ``check_gate`` are the two tolerances: the per-row
  bound ``|y - y_ref| <= 1e-5 * ||w_row||_2 * ||x||_2`` and the reference's
  own gate ``max|y - y_ref| / max|y_ref| <= 1e-5``
  (tests/test_correctness.py:21, src/bench.cu:229-240).
* ``quantize_x_q8_1`` / ``matvec_q8_1_ref`` restate the opt-in q8_1 activation
  path, which the reference names but does not implement (README.md:208-210,
  286-292: ggml's q8_1 route): x is rounded to int8 per 32-element block
  (``amax = max|x|``, ``id = fp32(127 / amax)``, ``dx = fp32(amax / 127)``,
  ``q = rint(fp32(x * id))``), then ``y = sum_b dw * dx * sum_j w_j q_j`` with
  exact integer block dots and a float64 combination.  Parity of that path
  is against this restatement (unpinned: no golden vectors exist for it);
  its distance to ``matvec_ref`` is the rounding of x, not a kernel error.
* ``to_aos`` / ``from_aos`` restate the ggml block byte layout
  (src/qgemv_kernels.cuh:21-26: little-endian fp16 ``d`` then the quants) and
  the AoS<->SoA repack of src/bench.cu:300-314.

Inputs are finite fp32 weights: the reference's float -> int conversion of a
NaN or infinity is undefined behaviour in C, so non-finite weights are outside
the contract on both sides.

Parity pin: every function here is checked against golden vectors produced
by the reference's own python/qformats.py (tests/golden/make_golden.py) and,
where it was built, against the reference's C++ quantizers and float64
matvec compiled from src/bench.cu (oracle/ref_shim.cu).
"""

from __future__ import annotations

import numpy as np

QK = 32
Q8_BLOCK_BYTES = 34
Q4_BLOCK_BYTES = 18
TOL = 1e-5


def _blocks(W: np.ndarray) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.float32)
    if W.ndim != 2 or W.shape[1] % QK:
        raise ValueError(f"W must be [M, K] with K % {QK} == 0, got {W.shape}")
    M, K = W.shape
    return W.reshape(M, K // QK, QK)


def quantize_q8_0(W: np.ndarray):
    """qformats.py:17-25. Returns (q int8 [M,K], d float16 [M,K/32])."""
    Wb = _blocks(W)
    M, nb, _ = Wb.shape
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        amax = np.abs(Wb).max(axis=2)
        d = (amax / np.float32(127.0)).astype(np.float32)
        idv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, np.float32(1.0)),
                       np.float32(0.0)).astype(np.float32)
        prod = (Wb * idv[:, :, None]).astype(np.float32)
        q = np.clip(np.rint(prod), -127, 127).astype(np.int8)
    return q.reshape(M, nb * QK), d.astype(np.float16)


def quantize_q4_0(W: np.ndarray):
    """qformats.py:28-40. Returns (packed uint8 [M,K/2], d float16 [M,K/32])."""
    Wb = _blocks(W)
    M, nb, _ = Wb.shape
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        idx = np.argmax(np.abs(Wb), axis=2)
        mx = np.take_along_axis(Wb, idx[:, :, None], axis=2)[:, :, 0]
        d = (mx / np.float32(-8.0)).astype(np.float32)
        nz = d != 0
        idv = np.where(nz, np.float32(1.0) / np.where(nz, d, np.float32(1.0)),
                       np.float32(0.0)).astype(np.float32)
        t = (Wb * idv[:, :, None]).astype(np.float32)
        t = (t + np.float32(8.5)).astype(np.float32)
        # float -> int32 truncates toward zero, as Tensor.to(torch.int32) does.
        q = np.clip(t.astype(np.int32), 0, 15).astype(np.uint8)
    packed = (q[:, :, :16] | (q[:, :, 16:] << 4)).astype(np.uint8)
    return packed.reshape(M, nb * QK // 2), d.astype(np.float16)


def dequant_q8_0(q: np.ndarray, d: np.ndarray) -> np.ndarray:
    """qformats.py:43-46, float32."""
    M, K = q.shape
    return (q.reshape(M, K // QK, QK).astype(np.float32)
            * d.astype(np.float32)[:, :, None]).reshape(M, K)


def q4_nibbles(packed: np.ndarray) -> np.ndarray:
    """Unpack q4_0 bytes to the 32 quants of each block (0..15), ggml order."""
    M, Kh = packed.shape
    p = packed.reshape(M, Kh // (QK // 2), QK // 2)
    return np.concatenate([p & 0x0F, p >> 4], axis=2).reshape(M, Kh * 2)


def dequant_q4_0(packed: np.ndarray, d: np.ndarray) -> np.ndarray:
    """qformats.py:49-56, float32."""
    M, Kh = packed.shape
    K = Kh * 2
    w = q4_nibbles(packed).astype(np.float32) - np.float32(8.0)
    return (w.reshape(M, K // QK, QK) * d.astype(np.float32)[:, :, None]).reshape(M, K)


def dequant_f64(fmt: str, q: np.ndarray, d: np.ndarray) -> np.ndarray:
    """Dequantize in float64 (exact: int8 or nibble times an fp16 scale)."""
    if fmt == "q8_0":
        M, K = q.shape
        vals = q.astype(np.float64)
    elif fmt == "q4_0":
        M, K = q.shape[0], q.shape[1] * 2
        vals = q4_nibbles(q).astype(np.float64) - 8.0
    else:
        raise ValueError(fmt)
    return (vals.reshape(M, K // QK, QK) * d.astype(np.float64)[:, :, None]).reshape(M, K)


def matvec_ref(fmt: str, q: np.ndarray, d: np.ndarray, X: np.ndarray) -> np.ndarray:
    """float64 dequant-matvec over the quantized bytes (bench.cu:75-111).

    ``X`` is ``[K]`` or ``[N, K]`` (one activation vector per row); the result
    is ``[M]`` or ``[N, M]`` in float64.
    """
    Wd = dequant_f64(fmt, q, d)
    X64 = np.asarray(X, dtype=np.float64)
    if X64.ndim == 1:
        return Wd @ X64
    return X64 @ Wd.T


def quantize_x_q8_1(X: np.ndarray):
    """Activations -> (int8 quants as int32 [..., K], fp32 scales [..., K/32]).

    Per 32-element block: ``amax = max|x|``; ``id = fp32(127 / amax)`` and
    ``dx = fp32(amax / 127)`` (correctly rounded fp32 divisions; an all-zero
    block gives ``id = dx = 0``); ``q = rint(fp32(x * id))`` (round half to
    even), so ``|q| <= 127``.
    """
    X = np.asarray(X, dtype=np.float32)
    K = X.shape[-1]
    B = X.reshape(X.shape[:-1] + (K // QK, QK))
    amax = np.abs(B).max(axis=-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        idv = np.where(amax > 0, np.float32(127.0) / amax, np.float32(0.0)).astype(np.float32)
        dx = (amax / np.float32(127.0)).astype(np.float32)
        prod = (B * idv[..., None]).astype(np.float32)
    q = np.rint(np.where(np.isfinite(prod), prod, 0.0)).astype(np.int32)
    return q.reshape(X.shape), dx


def matvec_q8_1_ref(fmt: str, q: np.ndarray, d: np.ndarray, X: np.ndarray) -> np.ndarray:
    """The opt-in q8_1 path: ``y[r] = sum_b dw[r,b] * dx[b] * sum_j w[r,b,j] * xq[b,j]``.

    The integer block dots are exact (int64) and the combination float64; the
    result is ``[M]`` or ``[N, M]`` like ``matvec_ref``.
    """
    if fmt == "q8_0":
        M, K = q.shape
        W = q.astype(np.int64)
    elif fmt == "q4_0":
        M, K = q.shape[0], q.shape[1] * 2
        W = q4_nibbles(q).astype(np.int64) - 8
    else:
        raise ValueError(fmt)
    nb = K // QK
    Wb = W.reshape(M, nb, QK)
    d64 = d.astype(np.float64)
    X2 = np.atleast_2d(np.asarray(X, dtype=np.float32))
    xq, dx = quantize_x_q8_1(X2)
    out = np.empty((X2.shape[0], M), dtype=np.float64)
    for n in range(X2.shape[0]):
        S = np.einsum("mbj,bj->mb", Wb, xq[n].reshape(nb, QK).astype(np.int64))
        with np.errstate(invalid="ignore"):
            out[n] = (S.astype(np.float64) * d64 * dx[n].astype(np.float64)[None, :]).sum(axis=1)
    return out[0] if np.asarray(X).ndim == 1 else out


def row_norms(fmt: str, q: np.ndarray, d: np.ndarray) -> np.ndarray:
    """||w_row||_2 of the dequantized rows, float64."""
    Wd = dequant_f64(fmt, q, d)
    return np.sqrt((Wd * Wd).sum(axis=1))


def check_rowwise(y, y_ref, wnorm, X, tol: float = TOL):
    """Per-row bound |y - y_ref| <= tol * ||w_row|| * ||x||.  Returns (ok, worst ratio)."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    X64 = np.asarray(X, dtype=np.float64)
    if X64.ndim == 1:
        bound = tol * wnorm * np.sqrt((X64 * X64).sum())
    else:
        bound = tol * wnorm[None, :] * np.sqrt((X64 * X64).sum(axis=1))[:, None]
    err = np.abs(y - y_ref)
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = np.where(bound > 0, err / np.where(bound > 0, bound, 1.0),
                         np.where(err > 0, np.inf, 0.0))
    worst = float(ratio.max()) if ratio.size else 0.0
    return bool(np.all(err <= bound)), worst


def check_gate(y, y_ref, tol: float = TOL):
    """Reference gate: max|y - y_ref| / max|y_ref| <= tol (bench.cu:229-240)."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    max_abs = float(np.abs(y - y_ref).max()) if y.size else 0.0
    scale = float(np.abs(y_ref).max()) if y.size else 0.0
    max_rel = max_abs / scale if scale > 0 else (0.0 if max_abs == 0 else np.inf)
    return max_rel <= tol, max_abs, max_rel


def to_aos(fmt: str, q: np.ndarray, d: np.ndarray) -> np.ndarray:
    """SoA planes -> ggml blocks, uint8 [M, K/32, 34|18] (d little-endian first)."""
    d = np.ascontiguousarray(d, dtype=np.float16)
    M, nb = d.shape
    qb = q.reshape(M, nb, -1).view(np.uint8)
    db = d.view(np.uint8).reshape(M, nb, 2)
    return np.ascontiguousarray(np.concatenate([db, qb], axis=2))


def from_aos(fmt: str, blocks: np.ndarray):
    """ggml blocks uint8 [M, K/32, 34|18] -> (q, d) SoA planes."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    M, nb, bs = blocks.shape
    d = np.ascontiguousarray(blocks[:, :, :2]).view(np.float16).reshape(M, nb)
    qs = np.ascontiguousarray(blocks[:, :, 2:])
    if fmt == "q8_0":
        assert bs == Q8_BLOCK_BYTES
        return qs.view(np.int8).reshape(M, nb * QK), d
    assert bs == Q4_BLOCK_BYTES
    return qs.reshape(M, nb * QK // 2), d


def block_bytes(fmt: str) -> int:
    return Q8_BLOCK_BYTES if fmt == "q8_0" else Q4_BLOCK_BYTES


def weight_bytes(fmt: str, M: int, K: int) -> int:
    """Bytes of a quantized [M, K] matrix: M*K*(34|18)/32."""
    return M * (K // QK) * block_bytes(fmt)


def dequant_torch(fmt: str, q, d):
    """The reference's CPU GEMV operand, ``dequant_q8_0 / dequant_q4_0`` of
    python/qformats.py:43-56, restated with torch CPU tensors (fp32): the
    quants times their block's fp16 scale, q4_0 nibbles (low -> j, high ->
    j + 16) minus 8.  ``dequant_torch(fmt, q, d) @ x`` is the reference's CPU
    path (python/triton_qgemv.py:135,154); used only as a timed baseline."""
    import torch
    q = torch.as_tensor(q)
    d = torch.as_tensor(d)
    M = q.shape[0]
    if fmt == "q8_0":
        w = q.reshape(M, -1, QK).to(torch.float32)
    else:
        b = q.reshape(M, -1, QK // 2)
        w = torch.cat([b & 0x0F, b >> 4], dim=2).to(torch.float32) - 8.0
    return (w * d.to(torch.float32).unsqueeze(2)).reshape(M, -1)


def quantize(fmt: str, W: np.ndarray):
    return quantize_q8_0(W) if fmt == "q8_0" else quantize_q4_0(W)


def dequant(fmt: str, q, d):
    return dequant_q8_0(q, d) if fmt == "q8_0" else dequant_q4_0(q, d)
