"""CPU oracle for the csaq-quant quantised hot path (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the arithmetic of csaq-quant v0.5.9 for the
functions on the quantised hot path. Only ``tests/``, ``__graft_entry__.smoke``
and the CPU-baseline legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline; the product path (the ``csaq`` package
under ``csaq-quant_b200/``) never calls it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by the reference itself (``tests/golden/
make_goldens.py`` imports csaq-quant and records its outputs).

Float rules followed exactly (all in IEEE fp32, one rounding per op):
* ``torch.round`` is round-half-to-even (``np.rint``);
* division by a Python int on a CPU tensor is a true IEEE division;
* a float32 tensor combined with a Python float keeps float32 (the scalar is
  rounded to float32 first);
* ``.to(torch.int32)`` of NaN on x86 yields INT32_MIN, and uint8 casts keep
  the low byte.
"""

from __future__ import annotations

import warnings
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

F32 = np.float32
INT32_MIN = np.int32(-2147483648)


def _to_i32(v: np.ndarray) -> np.ndarray:
    """torch ``.to(torch.int32)`` on x86: truncation, NaN/out-of-range -> INT32_MIN."""
    v = np.asarray(v, dtype=F32)
    out = np.full(v.shape, INT32_MIN, dtype=np.int32)
    ok = np.isfinite(v) & (v >= -2147483648.0) & (v < 2147483648.0)
    out[ok] = np.trunc(v[ok]).astype(np.int64).astype(np.int32)
    return out


def _clamp(v: np.ndarray, lo: float, hi: float) -> np.ndarray:
    """torch.clamp: NaN propagates."""
    return np.where(np.isnan(v), v, np.minimum(np.maximum(v, F32(lo)), F32(hi))).astype(F32)


# ─── csaq/kernels.py:495-508 ────────────────────────────────────────────────
def compute_scale_zp(w_min: np.ndarray, w_max: np.ndarray, bits: int):
    """Asymmetric scale / zero point (csaq/kernels.py:495-508)."""
    n_levels = 2 ** bits - 1
    w_min = np.asarray(w_min, dtype=F32)
    w_max = np.asarray(w_max, dtype=F32)
    w_max = np.where(w_max > w_min, w_max, (w_min + F32(1e-8)).astype(F32)).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = ((w_max - w_min).astype(F32) / F32(n_levels)).astype(F32)
        zp_f = np.rint((-w_min).astype(F32) / scale).astype(F32)
    zp = _to_i32(_clamp(zp_f, 0, n_levels))
    return scale, zp


# ─── csaq/kernels.py:511-523 ────────────────────────────────────────────────
def quantize_rows(W: np.ndarray, scale: np.ndarray, zp: np.ndarray, bits: int) -> np.ndarray:
    """q = clamp(round(W/scale + zp), 0, 2^b-1) as int32 (csaq/kernels.py:511-523)."""
    n_levels = 2 ** bits - 1
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        v = (np.asarray(W, F32) / scale).astype(F32)
        v = (v + zp.astype(F32)).astype(F32)
        v = np.rint(v).astype(F32)
    return _to_i32(_clamp(v, 0, n_levels))


# ─── csaq/kernels.py:526-536 ────────────────────────────────────────────────
def float_to_int(W: np.ndarray, scales: np.ndarray, zps: np.ndarray, bits: int) -> np.ndarray:
    """Row-wise requantisation of a reconstructed W (csaq/kernels.py:526-536)."""
    n_levels = 2 ** bits - 1
    sc = np.asarray(scales, F32)[:, None]
    zp = np.asarray(zps).astype(F32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        v = (np.asarray(W, F32) / sc).astype(F32)
        v = np.rint((v + zp).astype(F32)).astype(F32)
    return _to_i32(_clamp(v, 0, n_levels))


# ─── csaq/kernels.py:539-569 ────────────────────────────────────────────────
def pack(Wq: np.ndarray, bits: int) -> np.ndarray:
    """Pack int codes to uint8 (csaq/kernels.py:539-569).

    4-bit: even column in the low nibble, odd column in the high nibble.
    2-bit: column 4j+t at bits 2t of byte j. 8-bit: low byte.
    """
    q = np.asarray(Wq).astype(np.int64).astype(np.uint8)  # low byte, like .to(uint8)
    if bits == 8:
        return np.ascontiguousarray(q)
    rows, cols = q.shape
    if bits == 4:
        if cols % 2:
            q = np.pad(q, ((0, 0), (0, 1)))
        return ((q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    if bits == 2:
        pad = (4 - cols % 4) % 4
        if pad:
            q = np.pad(q, ((0, 0), (0, pad)))
        return ((q[:, 0::4] & 3) | ((q[:, 1::4] & 3) << 2) | ((q[:, 2::4] & 3) << 4)
                | ((q[:, 3::4] & 3) << 6)).astype(np.uint8)
    raise ValueError(f"Unsupported bits for packing: {bits}")


# ─── csaq/kernels.py:572-600 ────────────────────────────────────────────────
def unpack(packed: np.ndarray, bits: int, rows: int, cols: int) -> np.ndarray:
    """Inverse of :func:`pack`; int32 (rows, cols) (csaq/kernels.py:572-600)."""
    p = np.asarray(packed, dtype=np.uint8)
    if bits == 8:
        return p.reshape(rows, cols).astype(np.int32)
    if bits == 4:
        out = np.zeros((rows, p.shape[1] * 2), np.int32)
        out[:, 0::2] = p & 0xF
        out[:, 1::2] = (p >> 4) & 0xF
        return out[:, :cols]
    if bits == 2:
        out = np.zeros((rows, p.shape[1] * 4), np.int32)
        for t in range(4):
            out[:, t::4] = (p >> (2 * t)) & 3
        return out[:, :cols]
    raise ValueError(f"Unsupported bits for unpacking: {bits}")


def _assert_supported(bits: int) -> None:
    """csaq/kernels.py:488-492."""
    if bits not in (2, 4, 8):
        raise ValueError(f"[CSAQ kernels] bits={bits} not supported.  Use 2, 4, 8, or 16.")


class QW:
    """Numpy mirror of ``QuantizedWeight`` (csaq/kernels.py:34-70)."""

    def __init__(self, qdata, scales, zero_points, bits, rows, cols, group_size=-1,
                 shared_scale=False):
        self.qdata, self.scales, self.zero_points = qdata, scales, zero_points
        self.bits, self.rows, self.cols = bits, rows, cols
        self.group_size, self.shared_scale = group_size, shared_scale

    def dequantize(self) -> np.ndarray:
        return dequantize(self)


def _as_f32(W) -> np.ndarray:
    """``W.detach().float()``: exact widening from fp16/bf16/fp32."""
    return np.asarray(W).astype(F32)


# ─── csaq/kernels.py:77-158 ─────────────────────────────────────────────────
def quantize_per_channel(W: np.ndarray, bits: int, group_size: int = -1) -> QW:
    """Per-channel or per-group asymmetric quantisation (csaq/kernels.py:77-158).

    ``W`` may be float16 (numpy) or float32; bfloat16 callers pass the exact
    float32 widening. Per-group pads the last group with zeros, and the pad
    zeros take part in the group's min/max (csaq/kernels.py:130-137).
    """
    W = np.asarray(W)
    if bits == 16:
        fp16 = W.astype(np.float16)
        rows, cols = W.shape
        return QW(fp16.view(np.uint8).reshape(rows, cols * 2).copy(),
                  np.ones(rows, F32), np.zeros(rows, np.int32), 16, rows, cols, group_size)
    _assert_supported(bits)
    W32 = _as_f32(W)
    rows, cols = W32.shape
    if group_size == -1 or group_size >= cols:
        w_min = W32.min(axis=1)
        w_max = W32.max(axis=1)
        scales, zps = compute_scale_zp(w_min, w_max, bits)
        Wq = quantize_rows(W32, scales[:, None], zps[:, None], bits)
        return QW(pack(Wq, bits), scales, zps, bits, rows, cols, -1)
    n_groups = (cols + group_size - 1) // group_size
    pad = n_groups * group_size - cols
    if pad:
        W32 = np.pad(W32, ((0, 0), (0, pad)))
    Wg = W32.reshape(rows, n_groups, group_size)
    w_min = Wg.min(axis=2)
    w_max = Wg.max(axis=2)
    scales, zps = compute_scale_zp(w_min, w_max, bits)
    Wq = quantize_rows(Wg.reshape(rows * n_groups, group_size),
                       scales.reshape(-1, 1), zps.reshape(-1, 1), bits)
    Wq = Wq.reshape(rows, n_groups * group_size)[:, :cols]
    return QW(pack(Wq, bits), scales, zps, bits, rows, cols, group_size)


# ─── csaq/kernels.py:161-268 ────────────────────────────────────────────────
def quantize_shared_scale(W: np.ndarray, leader_row: np.ndarray, bits: int,
                          group_size: int = -1) -> QW:
    """Leader-row shared-scale quantisation (csaq/kernels.py:161-268)."""
    W = np.asarray(W)
    if bits == 16:
        fp16 = W.astype(np.float16)
        rows, cols = W.shape
        return QW(fp16.view(np.uint8).reshape(rows, cols * 2).copy(),
                  np.ones(rows, F32), np.zeros(rows, np.int32), 16, rows, cols,
                  group_size, True)
    _assert_supported(bits)
    W32 = _as_f32(W)
    L32 = _as_f32(leader_row)
    rows, cols = W32.shape
    if group_size == -1 or group_size >= cols:
        l_min = L32.min(keepdims=True)
        l_max = L32.max(keepdims=True)
        scale, zp = compute_scale_zp(l_min, l_max, bits)
        follower_range = float(np.abs(W32).max())
        leader_range = float(np.abs((l_max - l_min).astype(F32))[0])
        if leader_range > 0 and follower_range / leader_range > 4.0:
            warnings.warn(
                f"[CSAQ kernels] Follower row outlier: follower/leader range "
                f"ratio={follower_range / leader_range:.1f} (bits={bits}). "
                "Consider increasing group_size or clique_threshold.", stacklevel=2)
        Wq = quantize_rows(W32, scale[:, None], zp[:, None], bits)
        return QW(pack(Wq, bits), np.repeat(scale, rows), np.repeat(zp, rows), bits,
                  rows, cols, -1, True)
    n_groups = (cols + group_size - 1) // group_size
    pad = n_groups * group_size - cols
    L_pad = np.pad(L32, (0, pad)).reshape(n_groups, group_size)
    W_pad = np.pad(W32, ((0, 0), (0, pad))).reshape(rows, n_groups, group_size)
    scales, zp = compute_scale_zp(L_pad.min(axis=1), L_pad.max(axis=1), bits)
    Wq = quantize_rows(W_pad.reshape(rows * n_groups, group_size),
                       np.tile(scales, rows).reshape(-1, 1),
                       np.tile(zp, rows).reshape(-1, 1), bits)
    Wq = Wq.reshape(rows, n_groups * group_size)[:, :cols]
    return QW(pack(Wq, bits), np.tile(scales, (rows, 1)), np.tile(zp, (rows, 1)), bits,
              rows, cols, group_size, True)


# ─── csaq/kernels.py:603-619 ────────────────────────────────────────────────
def dequantize(qw: QW) -> np.ndarray:
    """fp32 reconstruction (csaq/kernels.py:603-619)."""
    if qw.bits == 16:
        return qw.qdata.view(np.float16).astype(F32).reshape(qw.rows, qw.cols)
    Wq = unpack(qw.qdata, qw.bits, qw.rows, qw.cols).astype(F32)
    sc = np.asarray(qw.scales, F32)
    zp = np.asarray(qw.zero_points).astype(F32)
    if qw.group_size == -1 or sc.ndim == 1:
        return ((Wq - zp[:, None]).astype(F32) * sc[:, None]).astype(F32)
    n_groups = sc.shape[1]
    gs = qw.cols // n_groups
    Wg = Wq.reshape(qw.rows, n_groups, gs)
    return ((Wg - zp[:, :, None]).astype(F32) * sc[:, :, None]).astype(F32).reshape(
        qw.rows, qw.cols)


def dequantize_grouped(qdata, scales, zps, bits, rows, cols, group_size) -> np.ndarray:
    """Per-group dequant that also handles a ragged last group.

    The reference reshapes (rows, cols) into (rows, G, cols // G), which only
    works when group_size divides cols (csaq/kernels.py:613-619). This helper
    gives the same values there and extends the rule (column c uses group
    c // group_size) to ragged widths.
    """
    if bits == 16:
        return qdata.view(np.float16).astype(F32).reshape(rows, cols)
    Wq = unpack(qdata, bits, rows, cols).astype(F32)
    sc = np.asarray(scales, F32).reshape(rows, -1)
    zp = np.asarray(zps).astype(F32).reshape(rows, -1)
    g = np.arange(cols) // (group_size if group_size > 0 else cols)
    return ((Wq - zp[:, g]).astype(F32) * sc[:, g]).astype(F32)


# ─── csaq/kernels.py:371-448 ────────────────────────────────────────────────
def from_cliques(W: np.ndarray, clique_list: Sequence[dict]) -> Tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """Buffers of ``CSAQLinear.from_cliques`` (csaq/kernels.py:371-448).

    Returns (weight_packed, weight_scales, weight_zp, dominant_bits).
    Every clique is quantised at the dominant bit-width with its leader's
    per-row (group_size -1) scale; uncovered rows are quantised per channel.
    """
    W32 = _as_f32(W)
    out_f, in_f = W32.shape
    bit_counts: Dict[int, int] = {}
    for c in clique_list:
        b = c.get("bits", 4)
        bit_counts[b] = bit_counts.get(b, 0) + len(c.get("rows", []))
    dominant = max(bit_counts, key=bit_counts.__getitem__)
    W_rec = np.zeros_like(W32)
    all_scales = np.ones(out_f, F32)
    all_zp = np.zeros(out_f, np.int32)
    covered = set()
    for c in clique_list:
        rows = list(c["rows"])
        qw = quantize_shared_scale(W32[rows], W32[c["leader"]], dominant, -1)
        W_rec[rows] = qw.dequantize()
        all_scales[rows] = qw.scales[:len(rows)]
        all_zp[rows] = qw.zero_points[:len(rows)]
        covered.update(rows)
    uncovered = [i for i in range(out_f) if i not in covered]
    if uncovered:
        qw = quantize_per_channel(W32[uncovered], dominant, -1)
        W_rec[uncovered] = qw.dequantize()
        all_scales[uncovered] = qw.scales[:len(uncovered)]
        all_zp[uncovered] = qw.zero_points[:len(uncovered)]
    if dominant == 16:
        raise ValueError("Unsupported bits for packing: 16")
    Wq = float_to_int(W_rec, all_scales, all_zp, dominant)
    return pack(Wq, dominant), all_scales, all_zp, dominant


# ─── csaq/kernels.py:450-475 ────────────────────────────────────────────────
def get_weight_fp32(weight_packed, weight_scales, weight_zp, bits, rows, cols) -> np.ndarray:
    """``CSAQLinear._get_weight_fp32`` (csaq/kernels.py:450-468), per-channel."""
    if bits == 16:
        return np.asarray(weight_packed).view(np.float16).astype(F32).reshape(rows, cols)
    Wq = unpack(weight_packed, bits, rows, cols).astype(F32)
    sc = np.asarray(weight_scales, F32).reshape(rows, -1)
    zp = np.asarray(weight_zp).astype(F32).reshape(rows, -1)
    W = ((Wq - zp).astype(F32) * sc).astype(F32)
    return np.nan_to_num(W, nan=0.0, posinf=65504.0, neginf=-65504.0).astype(F32)


def linear_ref(x: np.ndarray, W32: np.ndarray, bias: Optional[np.ndarray] = None) -> np.ndarray:
    """fp32 reference of ``F.linear(x, W) + bias`` (csaq/kernels.py:470-475),
    accumulated in float64 and rounded to fp32 (the comparison target of the
    GPU GEMV/GEMM, which accumulate in fp32)."""
    y = np.asarray(x, np.float64) @ np.asarray(W32, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return y.astype(F32)


def mixed_weight(W: np.ndarray, tier_rows: Dict[int, np.ndarray], group_size: int = 128) -> np.ndarray:
    """Tier-composed dequantised weight of a mixed-row layer.

    Each tier is ``quantize_per_channel(W[rows_t], bits, group_size)`` and its
    dequantisation (csaq/kernels.py:77-158, 603-619); 16-bit rows are the fp16
    cast (csaq/kernels.py:94-107).
    """
    W = np.asarray(W)
    out = np.zeros(W.shape, F32)
    for bits, rows in tier_rows.items():
        rows = np.asarray(rows, np.int64)
        if rows.size == 0:
            continue
        qw = quantize_per_channel(W[rows], bits, group_size)
        if bits == 16:
            out[rows] = qw.dequantize()
        else:
            out[rows] = dequantize_grouped(qw.qdata, qw.scales, qw.zero_points, bits,
                                           qw.rows, qw.cols, qw.group_size)
    return out


# ─── csaq/core.py:143-155 ───────────────────────────────────────────────────
def topk_mask(out: np.ndarray, salience_alpha: float = 1.0) -> np.ndarray:
    """Profiler forward-hook mask (csaq/core.py:143-155): per token, keep
    channels whose |o| >= the k-th largest |o| (ties kept),
    k = max(1, int(min(1, 0.1*alpha) * C))."""
    o = np.asarray(out)
    o = o.reshape(-1, o.shape[-1])
    C = o.shape[-1]
    frac = min(1.0, 0.1 * salience_alpha)
    k = max(1, int(frac * C))
    if k >= C:
        return np.ones(o.shape, dtype=bool)
    a = np.abs(o)
    thr = -np.partition(-a, k - 1, axis=1)[:, k - 1:k]
    return a >= thr


def threshold_mask(act: np.ndarray, thr: float = 0.5) -> np.ndarray:
    """Mask = act > thr, compared in the activation's own dtype."""
    a = np.asarray(act)
    return a > a.dtype.type(thr)


# ─── csaq/core.py:240-287 ───────────────────────────────────────────────────
def coact_counts(mask: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Intersection counts I = mask^T mask and f = column sums (csaq/core.py:261-263)."""
    m = np.asarray(mask, dtype=F32)
    inter = (m.T @ m).astype(np.int64)
    f = m.sum(axis=0).astype(np.int64)
    return inter, f


def jaccard(inter: np.ndarray, f: np.ndarray) -> np.ndarray:
    """J = I / clamp(f_i + f_j - I, min=1) in fp32 (csaq/core.py:263-265)."""
    I = inter.astype(F32)
    ff = f.astype(F32)
    union = ((ff[:, None] + ff[None, :]).astype(F32) - I).astype(F32)
    union = np.maximum(union, F32(1.0))
    return (I / union).astype(F32)


def greedy_cliques(J: np.ndarray, threshold: float) -> List[List[int]]:
    """Seed-order greedy partition (csaq/core.py:268-285)."""
    n = J.shape[0]
    thr = F32(threshold)
    visited = np.zeros(n, dtype=bool)
    cliques: List[List[int]] = []
    for i in range(n):
        if visited[i]:
            continue
        similar = np.nonzero(J[i] >= thr)[0]
        clique = [int(j) for j in similar if not visited[j]]
        if i not in clique:
            clique.insert(0, i)
        cliques.append(clique)
        visited[np.asarray(clique, dtype=np.int64)] = True
    return cliques


def build_cliques(mask: np.ndarray, threshold: float) -> List[List[int]]:
    inter, f = coact_counts(mask)
    return greedy_cliques(jaccard(inter, f), threshold)


def cliques_from_labels(labels: np.ndarray) -> List[List[int]]:
    """Clique lists from a per-channel clique label in seed order."""
    order = np.argsort(labels, kind="stable")
    bounds = np.flatnonzero(np.diff(labels[order])) + 1
    return [g.tolist() for g in np.split(order, bounds)]


# ─── csaq/core.py:204-210, 232-233 ──────────────────────────────────────────
def salience_accumulate(W: np.ndarray, grads: Sequence[np.ndarray]) -> np.ndarray:
    """sal = sum_s |G_s * W| / n_samples in fp32 (csaq/core.py:204-210, 232-233)."""
    W32 = _as_f32(W)
    acc = np.zeros(W32.shape, F32)
    for G in grads:
        acc += np.abs(_as_f32(G) * W32)
    return (acc / F32(max(len(grads), 1))).astype(F32)


# ─── csaq/core.py:294-361 ───────────────────────────────────────────────────
def solve_clique_budget(salience: Dict[str, np.ndarray], cliques: Dict[str, List[List[int]]],
                        target_bits: float, bit_options: Sequence[int], protection_floor: float):
    """Greedy bit-budget solver (csaq/core.py:294-361). Returns
    (budget, tier_stats, actual_avg_bits); budget[layer] is a list of dicts
    with rows, bits, leader, salience, elems."""
    all_c = []
    options = sorted(bit_options)
    min_bits = options[0]
    for name, layer_cliques in cliques.items():
        s = np.asarray(salience[name], F32)
        for c in layer_cliques:
            sub = s[c]
            row_sal = sub.sum(axis=1, dtype=F32)
            leader_idx = int(np.argmax(row_sal))
            all_c.append({"layer": name, "rows": c, "salience": float(sub.sum(dtype=F32)),
                          "elems": len(c) * s.shape[1], "bits": min_bits,
                          "leader": c[leader_idx]})
    if not all_c:
        return {}, {}, float(target_bits)
    total = sum(c["elems"] for c in all_c)
    current = sum(c["elems"] * c["bits"] for c in all_c)
    target_total = target_bits * total
    all_c.sort(key=lambda x: x["salience"] / max(x["elems"], 1), reverse=True)
    n_protect = max(1, int(protection_floor * len(all_c)))
    for c in all_c[:n_protect]:
        floor_bits = max(c["bits"], min(8, max(options)))
        if floor_bits > c["bits"] and floor_bits in options:
            current += (floor_bits - c["bits"]) * c["elems"]
            c["bits"] = floor_bits
    for c in all_c:
        for b in options:
            if b <= c["bits"]:
                continue
            cost = (b - c["bits"]) * c["elems"]
            if current + cost <= target_total:
                current += cost
                c["bits"] = b
            else:
                break
    budget: Dict[str, list] = {}
    stats: Dict[str, int] = {}
    for c in all_c:
        budget.setdefault(c["layer"], []).append(c)
        stats[f"int{c['bits']}"] = stats.get(f"int{c['bits']}", 0) + c["elems"]
    return budget, stats, current / max(total, 1)


# ─── csaq/core.py:393-398 ───────────────────────────────────────────────────
def protected_rows(row_salience: np.ndarray, protection_floor: float) -> np.ndarray:
    """Sorted top-salience rows kept in fp16 for the verify pass (csaq/core.py:393-398)."""
    n = row_salience.shape[0]
    n_protect = max(1, int(protection_floor * n))
    idx = np.argsort(-np.asarray(row_salience, np.float64), kind="stable")[:n_protect]
    return np.sort(idx)


# ─── csaq/inference.py (corrected greedy self-speculation) ──────────────────
def greedy_accept(draft_ids: Sequence[int], verify_argmax: Sequence[int]) -> Tuple[int, List[int]]:
    """Greedy acceptance of one speculative block.

    ``verify_argmax[k]`` is the verifier's argmax after consuming the context
    plus draft tokens ``draft_ids[:k]``; len(verify_argmax) = K + 1. Returns
    (n_new, tokens): the accepted prefix, then the verifier's correction or
    its bonus token. This fixes the off-by-one of csaq/inference.py:486,
    which compares draft token k with the verifier's position k+1.
    """
    out: List[int] = []
    for k, d in enumerate(draft_ids):
        v = int(verify_argmax[k])
        if v == int(d):
            out.append(v)
        else:
            out.append(v)
            return len(out), out
    out.append(int(verify_argmax[len(draft_ids)]))
    return len(out), out


def spearman_rho(ranks: np.ndarray, prev_ranks: np.ndarray) -> float:
    """Spearman rho of two rank vectors (csaq/core.py:218-222)."""
    n = float(ranks.size)
    d = ranks.astype(F32) - prev_ranks.astype(F32)
    return 1.0 - (6.0 * float((d.astype(F32) ** 2).sum(dtype=F32))) / (n * (n ** 2 - 1))
