"""CPU reference computations for the hot-path ops (test infrastructure).

* ``gemv_ref``  -- ``y = x @ deq(W)^T`` (``tests/test_bolt_ops.py:237-238``), accumulated in fp64.
* ``moe_ref``   -- the per-(row, expert) relu^2 MoE loop (``tests/test_bolt_ops.py:253-259``) with
  the op's bf16 rounding points: h = bf16(z.W1), h = bf16(relu(h)^2), p = bf16(h.W2),
  out = bf16(sum_j w_j p_j) with the sum in fp32 over j ascending (``src/bolt_ops.cu:627-662``).
* ``route_ref`` -- sigmoid router with bf16-rounded gate weights (``src/bolt_ops.cu:399-404``),
  bias-corrected top-k with ties to the lower index (``src/bolt_ops.cu:489``), weights
  ``s / (sum s + 1e-20) * scale`` (``src/bolt_ops.cu:505-508``); logits in fp64.
* ``embed_ref`` -- Q8Embed: rows ``ids`` of a Q8_0 table dequantised and rounded to bf16, ids
  outside [0, vocab) reading row 0 (``src/bolt_ops.cu:1645-1660``, ``:1674-1687``).
* ``rms_norm_ref`` -- RmsNorm / SkipRmsNorm: v = x or bf16(x + skip), y = bf16(bf16(gamma) * v *
  rsqrt(mean(v^2) + eps)) (``src/bolt_ops.cu:1692-1815``); mean in fp64, products in fp32.
* ``mamba_ref``  -- MambaStep: 4-tap causal conv + silu (activations rounded to bf16), the Mamba-2
  state recurrence and the gated group norm (``tests/test_bolt_ops.py:389-413``,
  ``src/bolt_ops.cu:68-301``), in fp64 from the bf16 / fp32 inputs.
* ``rel_l2``    -- the reference's metric ``||a-b|| / ||b||`` (``tests/test_bolt_ops.py:62-64``).
"""

from __future__ import annotations

import numpy as np

from .quants import bf16_round, bf16_to_f32


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))


def _x_f32(x) -> np.ndarray:
    x = np.asarray(x)
    if x.dtype == np.uint16:  # bf16 bit patterns
        return bf16_to_f32(x)
    return x.astype(np.float32)


def gemv_ref(x, w_deq: np.ndarray) -> np.ndarray:
    """x: [R, K] (bf16 bits as uint16, or float); w_deq: fp32 [N, K] -> fp64 [R, N]."""
    return _x_f32(x).astype(np.float64) @ np.asarray(w_deq, dtype=np.float64).T


def moe_ref(z, idx: np.ndarray, w: np.ndarray, d1: np.ndarray, d2: np.ndarray):
    """z: [R, H] bf16 bits; idx: [R, k] int32; w: [R, k] fp32; d1[e]: fp32 [I, H]; d2[e]: fp32 [H, I]
    (arrays indexed by expert, or dicts holding only the experts idx references).

    Returns (out_f32 [R, H] before the final bf16 rounding, h [R*k, I] fp32 holding bf16 values,
    part [R*k, H] fp32 holding bf16 values).  Only the experts referenced by idx are touched.
    """
    zf = _x_f32(z).astype(np.float64)
    R, k = idx.shape
    H = zf.shape[1]
    I = d1[int(idx[0, 0])].shape[0]
    out = np.zeros((R, H), dtype=np.float32)
    h_all = np.zeros((R * k, I), dtype=np.float32)
    p_all = np.zeros((R * k, H), dtype=np.float32)
    for t in range(R):
        for j in range(k):
            e = int(idx[t, j])
            h = bf16_round((zf[t] @ d1[e].astype(np.float64).T).astype(np.float32))
            h = bf16_round(np.maximum(h, np.float32(0)) ** 2)
            p = bf16_round((h.astype(np.float64) @ d2[e].astype(np.float64).T).astype(np.float32))
            out[t] += np.float32(w[t, j]) * p
            h_all[t * k + j] = h
            p_all[t * k + j] = p
    return out, h_all, p_all


def embed_ref(w_raw: np.ndarray, ids) -> np.ndarray:
    """w_raw: uint8 [vocab, row_bytes] Q8_0 table; ids: int64 of any shape -> fp32 [..., K] holding
    bf16 values.  Element value = fp32(fp16 d) * int8 q, one rounding to bf16."""
    from .quants import dequant_q8_0

    w_raw = np.asarray(w_raw, dtype=np.uint8)
    ids = np.asarray(ids, dtype=np.int64)
    vocab = w_raw.shape[0]
    flat = ids.reshape(-1)
    rows = np.where((flat < 0) | (flat >= vocab), 0, flat)
    K = w_raw.shape[1] // 34 * 32
    deq = dequant_q8_0(w_raw[rows]) if rows.size else np.zeros((0, K), np.float32)
    return bf16_round(deq.astype(np.float32)).reshape(*ids.shape, K)


def rms_norm_ref(x, gamma: np.ndarray, eps: float, skip=None):
    """x, skip: [R, H] bf16 bits (uint16); gamma: fp32 [H].  Returns (y fp32 [R, H] holding bf16
    values, v fp32 [R, H] holding the bf16 values normalised: x, or bf16(x + skip))."""
    v = _x_f32(x)
    if skip is not None:
        v = bf16_round(v + _x_f32(skip))  # fp32 add + bf16 rounding = bf16 rounding of the exact sum
    ms = (v.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    rs = (1.0 / np.sqrt(ms + np.float64(eps))).astype(np.float32)
    g = bf16_round(np.asarray(gamma, dtype=np.float32))
    y = bf16_round((g * v).astype(np.float32) * rs)
    return y, v


def route_ref(x, gate_w: np.ndarray, bias: np.ndarray, topk: int, scale: float, tie_eps: float = 1e-6):
    """x: [R, K] bf16 bits; gate_w: fp32 [E, K]; bias: fp32 [E].

    Returns (idx [R, topk] int32, weights [R, topk] fp64, scores [R, E] fp64, near_tie [R] bool).
    ``near_tie[r]`` marks rows whose k-th and (k+1)-th bias-corrected scores are closer than
    ``tie_eps``; their index set may legitimately differ under a different fp32 summation order.
    """
    xf = _x_f32(x).astype(np.float64)
    gw = bf16_round(np.asarray(gate_w, dtype=np.float32)).astype(np.float64)
    logits = xf @ gw.T
    scores = 1.0 / (1.0 + np.exp(-logits))
    val = scores + np.asarray(bias, dtype=np.float32).astype(np.float64)[None, :]
    R, E = val.shape
    order = np.lexsort((np.broadcast_to(np.arange(E), (R, E)), -val), axis=1)  # desc value, asc index
    idx = order[:, :topk].astype(np.int32)
    sel = np.take_along_axis(scores, idx, axis=1)
    weights = sel / (sel.sum(axis=1, keepdims=True) + 1e-20) * scale
    near = np.zeros(R, dtype=bool)
    if topk < E:
        vs = np.take_along_axis(val, order, axis=1)
        near = (vs[:, topk - 1] - vs[:, topk]) < tie_eps
    return idx, weights, scores, near


def _silu(v):
    return v / (1.0 + np.exp(-v))


def mamba_ref(proj, conv_state, ssm_state, conv_w, conv_b, dt_bias, a_neg, d_skip, norm_w, heads: int, n_groups: int,
              eps: float, tmin: float, hd: int = 64, ds: int = 128):
    """One MambaStep over R rows from one state.

    proj: [R, di + cd + heads] bf16 bits; conv_state: [cd, 3] bf16 bits; ssm_state: f32 [heads, ds, hd];
    conv_w: f32 [cd, 4] and conv_b f32 [cd] (bf16 values); dt_bias, a_neg, d_skip f32 [heads]; norm_w
    f32 [di].  Returns per-row lists: (y [R, di] fp64 before bf16 rounding, xbc [R, cd] fp32 holding
    bf16 values, ypre [R, di], conv_states [R] of [cd, 3], ssm_states [R] of [heads, ds, hd])."""
    pf = _x_f32(proj).astype(np.float64)
    R = pf.shape[0]
    di = heads * hd
    cd = di + 2 * n_groups * ds
    gate, xbc_in, dt = pf[:, :di], pf[:, di:di + cd], pf[:, di + cd:]
    inp = np.concatenate([_x_f32(conv_state).astype(np.float64).T, xbc_in], 0)  # [3 + R, cd]
    w = np.asarray(conv_w, np.float64)
    b = np.asarray(conv_b, np.float64)
    xbc = np.zeros((R, cd), np.float32)
    for r in range(R):
        acc = (inp[r:r + 4] * w.T).sum(0) + b
        xbc[r] = bf16_round(_silu(acc).astype(np.float32))
    conv_states = [inp[r + 1:r + 4].T.copy() for r in range(R)]
    xs, Bm, Cm = xbc[:, :di], xbc[:, di:di + n_groups * ds], xbc[:, di + n_groups * ds:]
    st = np.asarray(ssm_state, np.float64).copy()
    hpg = heads // n_groups
    ypre = np.zeros((R, di))
    states = []
    for r in range(R):
        raw = dt[r] + np.asarray(dt_bias, np.float64)
        dts = np.maximum(np.where(raw > 20.0, raw, np.log1p(np.exp(np.minimum(raw, 20.0)))), tmin)
        dA = np.exp(np.asarray(a_neg, np.float64) * dts)
        xh = xs[r].astype(np.float64).reshape(heads, hd)
        Bh = np.repeat(Bm[r].astype(np.float64).reshape(n_groups, ds), hpg, 0)
        Ch = np.repeat(Cm[r].astype(np.float64).reshape(n_groups, ds), hpg, 0)
        st = st * dA[:, None, None] + (dts[:, None] * xh)[:, None, :] * Bh[:, :, None]
        ypre[r] = ((st * Ch[:, :, None]).sum(1) + np.asarray(d_skip, np.float64)[:, None] * xh).reshape(di)
        states.append(st.copy())
    v = (ypre * _silu(gate)).reshape(R, n_groups, di // n_groups)
    v = v / np.sqrt((v ** 2).mean(-1, keepdims=True) + eps)
    y = v.reshape(R, di) * np.asarray(norm_w, np.float64)
    return y, xbc, ypre, conv_states, states
