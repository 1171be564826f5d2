"""csaq.kernels — quantisation primitives and the quantised linear, on B200.

Drop-in for csaq-quant's ``csaq/kernels.py``: same names, signatures, buffer
schemas and error behaviour. Every computation runs in the sm_100a library
(libcsaq_b200.so) through its C ABI; CPU tensors are accepted and the results
are returned on the caller's device, but the work itself is always done on the
GPU. There is no CPU fallback: without a CUDA device these functions raise.

Storage contract (csaq/kernels.py:1-18 of csaq-quant):
  bits 2/4/8 -> packed uint8 codes + fp32 scales + int32 zero points per
  (row, group); bits 16 -> fp16 bit pattern viewed as uint8.

Extension beyond the reference: ``CSAQLinear`` also holds *mixed-row* layers
(``from_tiers``), where each row tier (16/8/4/2 bits, per-group scales) is
stored exactly as ``quantize_per_channel(W[rows_t], bits, group_size)`` would
store it; and a verify mode that patches the fp16 rows of protected outputs in
the same kernel launch (self-speculative decoding).
"""

from __future__ import annotations

import ctypes
import warnings
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch
import torch.nn as nn

from . import _lib
from ._lib import CsaqTier, check, dtype_code, lib, ptr, stream_of

__all__ = [
    "QuantizedWeight", "quantize_per_channel", "quantize_shared_scale", "inject_csaq_linear",
    "CSAQLinear", "_pack", "_unpack", "_dequantize", "_float_to_int", "_assert_supported",
]


# ─────────────────────────────────────────────────────────────────────────────
# QuantizedWeight (csaq/kernels.py:34-70)
# ─────────────────────────────────────────────────────────────────────────────

@dataclass
class QuantizedWeight:
    """Packed weight buffer + dequantisation metadata (csaq/kernels.py:34-70)."""

    qdata: torch.Tensor
    scales: torch.Tensor
    zero_points: torch.Tensor
    bits: int
    rows: int
    cols: int
    group_size: int = -1
    shared_scale: bool = False

    def dequantize(self) -> torch.Tensor:
        return _dequantize(self)

    def element_size_bytes(self) -> float:
        return self.bits / 8.0

    def compression_ratio(self) -> float:
        return 32.0 / self.bits


# ─────────────────────────────────────────────────────────────────────────────
# helpers
# ─────────────────────────────────────────────────────────────────────────────

def _assert_supported(bits: int) -> None:
    """csaq/kernels.py:488-492."""
    if bits not in (2, 4, 8):
        raise ValueError(f"[CSAQ kernels] bits={bits} not supported.  Use 2, 4, 8, or 16.")


def _on_gpu(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t
    return t.to(_lib.cuda_device())


def _float_input(W: torch.Tensor) -> torch.Tensor:
    """``W.detach()`` as a CUDA tensor in a kernel dtype (fp32/fp16/bf16), unit
    column stride. Other float dtypes take the ``.float()`` of the reference."""
    W = _on_gpu(W.detach())
    if W.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        W = W.float()
    if W.dim() != 2:
        raise ValueError(f"expected a 2-D weight, got shape {tuple(W.shape)}")
    if W.stride(1) != 1 or W.stride(0) < W.shape[1]:
        W = W.contiguous()
    return W


def _n_groups(cols: int, group_size: int) -> int:
    if group_size == -1 or group_size <= 0 or group_size >= cols:
        return 1
    return (cols + group_size - 1) // group_size


def _packed_cols(cols: int, bits: int) -> int:
    return {8: cols, 4: (cols + 1) // 2, 2: (cols + 3) // 4, 16: cols * 2}[bits]


def _gpu_quant(W: torch.Tensor, bits: int, group_size: int):
    """(qdata, scales (rows, G), zps (rows, G)) for a CUDA 2-D float W."""
    rows, cols = W.shape
    G = _n_groups(cols, group_size)
    q = torch.empty(rows, _packed_cols(cols, bits), dtype=torch.uint8, device=W.device)
    s = torch.empty(rows, G, dtype=torch.float32, device=W.device)
    z = torch.empty(rows, G, dtype=torch.int32, device=W.device)
    if rows:
        check(lib().csaq_quant_pack(W.data_ptr(), dtype_code(W.dtype), rows, cols, W.stride(0), bits,
                                    group_size, q.data_ptr(), s.data_ptr(), z.data_ptr(),
                                    stream_of(W)), "quant_pack")
    return q, s, z


def _gpu_cast16(W: torch.Tensor) -> torch.Tensor:
    rows, cols = W.shape
    out = torch.empty(rows, cols, dtype=torch.float16, device=W.device)
    if rows * cols:
        check(lib().csaq_cast_f16(W.data_ptr(), dtype_code(W.dtype), rows, cols, W.stride(0),
                                  out.data_ptr(), stream_of(W)), "cast_f16")
    return out


def _gpu_group_scales(W: torch.Tensor, bits: int, group_size: int, absmax: bool = False):
    rows, cols = W.shape
    G = _n_groups(cols, group_size)
    s = torch.empty(rows, G, dtype=torch.float32, device=W.device)
    z = torch.empty(rows, G, dtype=torch.int32, device=W.device)
    a = torch.empty(rows, dtype=torch.float32, device=W.device) if absmax else None
    if rows:
        check(lib().csaq_group_scales(W.data_ptr(), dtype_code(W.dtype), rows, cols, W.stride(0), bits,
                                      group_size, s.data_ptr(), z.data_ptr(), ptr(a), stream_of(W)),
              "group_scales")
    return s, z, a


def _gpu_quant_rows(W: torch.Tensor, bits: int, group_size: int, s: torch.Tensor, z: torch.Tensor,
                    scale_mode: int, src_row: Optional[torch.Tensor] = None,
                    requant: bool = False) -> torch.Tensor:
    rows, cols = W.shape
    q = torch.empty(rows, _packed_cols(cols, bits), dtype=torch.uint8, device=W.device)
    if rows:
        s = s.contiguous()
        z = z.contiguous()
        check(lib().csaq_quant_pack_rows(W.data_ptr(), dtype_code(W.dtype), rows, cols, W.stride(0), bits,
                                         group_size, s.data_ptr(), z.data_ptr(), s.shape[-1],
                                         scale_mode, ptr(src_row), int(requant), q.data_ptr(),
                                         stream_of(W)), "quant_pack_rows")
    return q


# ─────────────────────────────────────────────────────────────────────────────
# Public API
# ─────────────────────────────────────────────────────────────────────────────

def quantize_per_channel(W: torch.Tensor, bits: int, group_size: int = -1) -> QuantizedWeight:
    """Asymmetric per-channel / per-group quantisation (csaq/kernels.py:77-158).

    Bit-exact with the reference: codes, scales and zero points are produced
    by the fused sm_100a quantise+pack kernel (or the two-pass kernels for
    ragged layouts). Results are returned on W's device.
    """
    dev = W.device
    rows, cols = W.shape
    if bits == 16:
        fp16 = _gpu_cast16(_float_input(W))
        return QuantizedWeight(
            qdata=fp16.view(torch.uint8).to(dev), scales=torch.ones(rows, dtype=torch.float32, device=dev),
            zero_points=torch.zeros(rows, dtype=torch.int32, device=dev), bits=16, rows=rows,
            cols=cols, group_size=group_size)
    _assert_supported(bits)
    Wg = _float_input(W)
    q, s, z = _gpu_quant(Wg, bits, group_size)
    if group_size == -1 or group_size >= cols:
        return QuantizedWeight(q.to(dev), s.view(rows).to(dev), z.view(rows).to(dev), bits, rows,
                               cols, -1)
    return QuantizedWeight(q.to(dev), s.to(dev), z.to(dev), bits, rows, cols, group_size)


def quantize_shared_scale(W: torch.Tensor, leader_row: torch.Tensor, bits: int,
                          group_size: int = -1) -> QuantizedWeight:
    """Leader-row shared-scale quantisation (csaq/kernels.py:161-268)."""
    dev = W.device
    rows, cols = W.shape
    if bits == 16:
        fp16 = _gpu_cast16(_float_input(W))
        return QuantizedWeight(
            qdata=fp16.view(torch.uint8).to(dev), scales=torch.ones(rows, dtype=torch.float32, device=dev),
            zero_points=torch.zeros(rows, dtype=torch.int32, device=dev), bits=16, rows=rows,
            cols=cols, group_size=group_size, shared_scale=True)
    _assert_supported(bits)
    Wg = _float_input(W)
    L = _float_input(leader_row.reshape(1, -1))
    if group_size == -1 or group_size >= cols:
        s, z, _ = _gpu_group_scales(L, bits, -1)
        _, _, amax = _gpu_group_scales(Wg, bits, -1, absmax=True)
        follower_range = float(amax.max()) if rows else 0.0
        Lf = L.float()
        leader_range = float((Lf.max() - Lf.min()).abs())
        if leader_range > 0 and follower_range / leader_range > 4.0:
            warnings.warn(
                f"[CSAQ kernels] Follower row outlier: follower/leader range "
                f"ratio={follower_range / leader_range:.1f} (bits={bits}). "
                "Consider increasing group_size or clique_threshold.", stacklevel=2)
        q = _gpu_quant_rows(Wg, bits, -1, s, z, scale_mode=1)
        return QuantizedWeight(q.to(dev), s.view(1).expand(rows).contiguous().to(dev),
                               z.view(1).expand(rows).contiguous().to(dev), bits, rows, cols, -1,
                               True)
    s, z, _ = _gpu_group_scales(L, bits, group_size)  # (1, G), zero-padded leader groups
    q = _gpu_quant_rows(Wg, bits, group_size, s, z, scale_mode=1)
    return QuantizedWeight(q.to(dev), s.expand(rows, -1).contiguous().to(dev),
                           z.expand(rows, -1).contiguous().to(dev), bits, rows, cols, group_size,
                           True)


def _pack(Wq: torch.Tensor, bits: int) -> torch.Tensor:
    """int codes -> packed uint8 (csaq/kernels.py:539-569)."""
    if bits not in (2, 4, 8):
        raise ValueError(f"Unsupported bits for packing: {bits}")
    dev = Wq.device
    q = _on_gpu(Wq).to(torch.int32).contiguous()
    rows, cols = q.shape
    out = torch.empty(rows, _packed_cols(cols, bits), dtype=torch.uint8, device=q.device)
    check(lib().csaq_pack(q.data_ptr(), bits, rows, cols, out.data_ptr(), stream_of(q)), "pack")
    return out.to(dev)


def _unpack(packed: torch.Tensor, bits: int, rows: int, cols: int) -> torch.Tensor:
    """packed uint8 -> int32 (rows, cols) (csaq/kernels.py:572-600)."""
    if bits not in (2, 4, 8):
        raise ValueError(f"Unsupported bits for unpacking: {bits}")
    dev = packed.device
    p = _on_gpu(packed).contiguous()
    out = torch.empty(rows, cols, dtype=torch.int32, device=p.device)
    check(lib().csaq_unpack(p.data_ptr(), bits, rows, cols, out.data_ptr(), stream_of(p)), "unpack")
    return out.to(dev)


def _float_to_int(W: torch.Tensor, scales: torch.Tensor, zps: torch.Tensor, bits: int) -> torch.Tensor:
    """Row-wise requantisation (csaq/kernels.py:526-536)."""
    dev = W.device
    Wg = _on_gpu(W).float().contiguous()
    s = _on_gpu(scales).float().contiguous()
    z = _on_gpu(zps).to(torch.int32).contiguous()
    rows, cols = Wg.shape
    out = torch.empty(rows, cols, dtype=torch.int32, device=Wg.device)
    check(lib().csaq_float_to_int(Wg.data_ptr(), s.data_ptr(), z.data_ptr(), bits, rows, cols,
                                  out.data_ptr(), stream_of(Wg)), "float_to_int")
    return out.to(dev)


def _dequant_raw(qdata: torch.Tensor, scales: Optional[torch.Tensor], zps: Optional[torch.Tensor],
                 bits: int, rows: int, cols: int, group_size: int, nan_to_num: bool = False,
                 out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    p = _on_gpu(qdata).contiguous()
    s = _on_gpu(scales).float().contiguous() if scales is not None else None
    z = _on_gpu(zps).to(torch.int32).contiguous() if zps is not None else None
    out = torch.empty(rows, cols, dtype=out_dtype, device=p.device)
    check(lib().csaq_dequant(p.data_ptr(), ptr(s), ptr(z), bits, rows, cols, group_size,
                             int(nan_to_num), dtype_code(out_dtype), out.data_ptr(), stream_of(p)),
          "dequant")
    return out


def _dequantize(qw: QuantizedWeight) -> torch.Tensor:
    """fp32 reconstruction (csaq/kernels.py:603-619)."""
    if qw.bits == 16:
        return _dequant_raw(qw.qdata, None, None, 16, qw.rows, qw.cols, -1).to(qw.qdata.device)
    gs = -1 if (qw.group_size == -1 or qw.scales.dim() == 1) else qw.cols // qw.scales.shape[1]
    if gs != -1 and qw.group_size > 0 and qw.cols % qw.group_size == 0:
        gs = qw.group_size
    return _dequant_raw(qw.qdata, qw.scales, qw.zero_points, qw.bits, qw.rows, qw.cols,
                        gs).to(qw.qdata.device)


def inject_csaq_linear(model: nn.Module, budget: dict, verbose: bool = True) -> nn.Module:
    """Replace the nn.Linear layers named in *budget* (csaq/kernels.py:271-300)."""
    replaced = 0
    for name, clique_list in budget.items():
        parent_name, _, child_name = name.rpartition(".")
        parent = model if not parent_name else _get_submodule(model, parent_name)
        if parent is None:
            continue
        child = getattr(parent, child_name, None)
        if not isinstance(child, nn.Linear):
            continue
        new_layer = CSAQLinear.from_cliques(child, clique_list, verbose=verbose)
        setattr(parent, child_name, new_layer)
        replaced += 1
    if verbose:
        print(f"[CSAQ] Replaced {replaced} nn.Linear layers with CSAQLinear.")
    return model


# ─────────────────────────────────────────────────────────────────────────────
# CSAQLinear
# ─────────────────────────────────────────────────────────────────────────────

# From this many tokens on, forward() uses the tcgen05 dequantise-GEMM (csaq_qgemm)
# instead of the decode GEMV (which re-reads the weights once per 16 tokens).
GEMM_MIN_TOKENS = 32


class _Tier:
    """One row tier as the GEMV reads it (kept alive for the ctypes descriptors)."""

    __slots__ = ("bits", "rows", "codes", "scales", "zps_u8", "group_size", "n_groups",
                 "n_verify")

    def __init__(self, bits, rows, codes, scales, zps_u8, group_size, n_groups, n_verify):
        self.bits, self.rows, self.codes = bits, rows, codes
        self.scales, self.zps_u8 = scales, zps_u8
        self.group_size, self.n_groups, self.n_verify = group_size, n_groups, n_verify


def _zps_u8(z: torch.Tensor) -> torch.Tensor:
    """uint8 zero points for the GEMV. Values lie in [0, 2^b-1]; INT32_MIN only
    occurs with scale 0, whose product is 0 whatever the zero point."""
    return z.clamp(0, 255).to(torch.uint8).contiguous()


class CSAQLinear(nn.Module):
    """Packed-weight replacement for ``nn.Linear`` (csaq/kernels.py:307-481).

    Uniform layers keep the reference buffers ``weight_packed`` (uint8),
    ``weight_scales`` (fp32) and ``weight_zp`` (int32). Mixed-row layers
    (``from_tiers``) hold one set of ``tier{b}_*`` buffers per bit-width.
    ``forward`` runs the sm_100a quantised GEMV/GEMM; it never materialises
    the dequantised weight.
    """

    def __init__(self, in_features: int, out_features: int, bits: int,
                 bias: Optional[torch.Tensor] = None, group_size: int = -1) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.bits = bits
        self.group_size = group_size
        if bits == 16:
            cols_packed = in_features * 2
        elif bits == 8:
            cols_packed = in_features
        elif bits == 4:
            cols_packed = (in_features + 1) // 2
        elif bits == 2:
            cols_packed = (in_features + 3) // 4
        else:
            cols_packed = 1
        n_groups = 1 if group_size == -1 else (in_features + group_size - 1) // group_size
        self.register_buffer("weight_packed", torch.zeros(out_features, cols_packed, dtype=torch.uint8))
        if n_groups == 1:
            self.register_buffer("weight_scales", torch.ones(out_features, dtype=torch.float32))
            self.register_buffer("weight_zp", torch.zeros(out_features, dtype=torch.int32))
        else:
            self.register_buffer("weight_scales", torch.ones(out_features, n_groups, dtype=torch.float32))
            self.register_buffer("weight_zp", torch.zeros(out_features, n_groups, dtype=torch.int32))
        if bias is not None:
            self.register_buffer("bias", bias.detach().clone())
        else:
            self.bias = None  # type: ignore[assignment]
        self.tier_bits: List[int] = []      # non-empty for mixed-row layers
        self.verify_mode: bool = False      # use the fp16 backups of protected rows
        self._gemv_cache: Dict = {}

    # ── state-dict compatibility (csaq/kernels.py:362-369) ───────────────────
    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        names = ["weight_packed", "weight_scales", "weight_zp", "_csaq_fp16_backup",
                 "_csaq_quant_stash", "_csaq_hi_rows"]
        for b in self.tier_bits:
            names += [f"tier{b}_rows", f"tier{b}_packed", f"tier{b}_scales", f"tier{b}_zp"]
        for attr in names:
            key = f"{prefix}{attr}"
            if key in state_dict:
                cur = getattr(self, attr, None)
                if cur is not None and cur.shape != state_dict[key].shape:
                    cur.resize_(state_dict[key].shape)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)
        self._gemv_cache.clear()

    def _apply(self, fn, recurse=True):
        self._gemv_cache = {}
        return super()._apply(fn, recurse)

    # ── construction ──────────────────────────────────────────────────────────
    @classmethod
    def from_cliques(cls, linear: nn.Linear, clique_list: list, verbose: bool = False) -> "CSAQLinear":
        """Quantise each clique with its leader's scale (csaq/kernels.py:371-448).

        All cliques use the layer's dominant bit-width (by row count); rows
        outside every clique are quantised per channel. The reconstruction is
        requantised with the per-row scale/zero point, exactly as the
        reference does. One fused launch per layer.
        """
        out_f, in_f = linear.out_features, linear.in_features
        bit_counts: Dict[int, int] = {}
        for c in clique_list:
            b = c.get("bits", 4)
            bit_counts[b] = bit_counts.get(b, 0) + len(c.get("rows", []))
        dominant = max(bit_counts, key=bit_counts.__getitem__)
        layer = cls(in_features=in_f, out_features=out_f, bits=dominant, bias=linear.bias)
        dev = linear.weight.device
        W = _float_input(linear.weight.data)
        if dominant == 16:
            raise ValueError("Unsupported bits for packing: 16")
        _assert_supported(dominant)
        src = torch.arange(out_f, dtype=torch.int64)
        groups = []
        for c in clique_list:
            rows = torch.as_tensor(list(c["rows"]), dtype=torch.int64)
            src[rows] = int(c["leader"])
            groups.append((rows, int(c["leader"])))
        s_row, z_row, amax = _gpu_group_scales(W, dominant, -1, absmax=True)
        src_d = src.to(torch.int32).to(W.device)
        packed = _gpu_quant_rows(W, dominant, -1, s_row, z_row, scale_mode=2, src_row=src_d,
                                 requant=True)
        srcl = src.to(W.device)
        scales = s_row.view(-1)[srcl].contiguous()
        zps = z_row.view(-1)[srcl].contiguous()
        # follower-outlier warnings of quantize_shared_scale (csaq/kernels.py:208-218)
        if groups:
            lead = torch.tensor([l for _, l in groups], device=W.device)
            WL = W[lead].float()
            lead_range = (WL.amax(dim=1) - WL.amin(dim=1)).abs().cpu()
            amax_c = amax.cpu()
            for (rows, _), lr in zip(groups, lead_range.tolist()):
                if rows.numel() == 0:
                    continue
                fr = float(amax_c[rows].max())
                if lr > 0 and fr / lr > 4.0:
                    warnings.warn(
                        f"[CSAQ kernels] Follower row outlier: follower/leader range "
                        f"ratio={fr / lr:.1f} (bits={dominant}). "
                        "Consider increasing group_size or clique_threshold.", stacklevel=2)
        layer.weight_packed = packed.to(dev)
        layer.weight_scales = scales.to(dev)
        layer.weight_zp = zps.to(dev)
        layer.bits = dominant
        if verbose:
            cr = 32.0 / dominant
            print(f"  [CSAQLinear] {out_f}×{in_f} → {dominant}-bit "
                  f"(compression {cr:.1f}×, memory ↓{(1.0 - 1.0 / cr) * 100:.0f}%)")
        del linear.weight
        return layer

    @classmethod
    def from_tiers(cls, linear: nn.Linear, tier_rows: Dict[int, torch.Tensor], group_size: int = 128,
                   protected_rows: Optional[torch.Tensor] = None) -> "CSAQLinear":
        """Mixed-row layer: rows of bit-width b are stored as
        ``quantize_per_channel(W[rows_b], b, group_size)`` (bit-exact per tier).

        ``protected_rows`` (sorted output rows) get an fp16 copy of their
        original weights for the verify pass; inside each tier they are
        stored last so the verify launch can skip them.
        """
        out_f, in_f = linear.out_features, linear.in_features
        dev = linear.weight.device
        W = _float_input(linear.weight.data)
        counts = {b: int(torch.as_tensor(r).numel()) for b, r in tier_rows.items()}
        dominant = max(counts, key=counts.__getitem__)
        layer = cls(in_features=in_f, out_features=out_f, bits=dominant, bias=linear.bias,
                    group_size=group_size)
        # the uniform buffers are unused by mixed layers
        layer.weight_packed = torch.zeros(0, dtype=torch.uint8, device=dev)
        layer.weight_scales = torch.zeros(0, dtype=torch.float32, device=dev)
        layer.weight_zp = torch.zeros(0, dtype=torch.int32, device=dev)
        covered = torch.zeros(out_f, dtype=torch.bool)
        prot = None
        if protected_rows is not None:
            prot = torch.zeros(out_f, dtype=torch.bool)
            prot[torch.as_tensor(protected_rows, dtype=torch.int64).cpu()] = True
        for b in sorted(tier_rows, reverse=True):
            rows = torch.sort(torch.as_tensor(tier_rows[b], dtype=torch.int64).cpu()).values
            if covered[rows].any():
                raise ValueError("tier rows overlap")
            covered[rows] = True
            if prot is not None:
                rows = torch.cat([rows[~prot[rows]], rows[prot[rows]]])
            Wr = W[rows.to(W.device)]
            if b == 16:
                codes = _gpu_cast16(Wr).view(torch.uint8)
                s = torch.ones(rows.numel(), 1, dtype=torch.float32, device=W.device)
                z = torch.zeros(rows.numel(), 1, dtype=torch.int32, device=W.device)
            else:
                _assert_supported(b)
                codes, s, z = _gpu_quant(Wr, b, group_size)
            layer.register_buffer(f"tier{b}_rows", rows.to(torch.int32).to(dev))
            layer.register_buffer(f"tier{b}_packed", codes.to(dev))
            layer.register_buffer(f"tier{b}_scales", s.to(dev))
            layer.register_buffer(f"tier{b}_zp", z.to(dev))
            layer.tier_bits.append(b)
        if not bool(covered.all()):
            raise ValueError("tier rows must cover every output row")
        if protected_rows is not None:
            hi = torch.sort(torch.as_tensor(protected_rows, dtype=torch.int64)).values.to(W.device)
            layer.set_protected_rows(hi, W[hi].to(torch.float16))
        del linear.weight
        return layer

    @classmethod
    def empty_tiers(cls, in_features: int, out_features: int, tiers: Dict[int, int], group_size: int = 128,
                    bias: Optional[torch.Tensor] = None) -> "CSAQLinear":
        """A mixed-row layer with zeroed tier buffers of the given row counts,
        to be filled by load_state_dict (the loader of exported models)."""
        dominant = max(tiers, key=tiers.__getitem__)
        layer = cls(in_features=in_features, out_features=out_features, bits=dominant, bias=bias,
                    group_size=group_size)
        layer.weight_packed = torch.zeros(0, dtype=torch.uint8)
        layer.weight_scales = torch.zeros(0, dtype=torch.float32)
        layer.weight_zp = torch.zeros(0, dtype=torch.int32)
        G = (in_features + group_size - 1) // group_size if group_size > 0 else 1
        for b in sorted(tiers, reverse=True):
            n = int(tiers[b])
            if b != 16:
                _assert_supported(b)
            g = 1 if b == 16 else G
            layer.register_buffer(f"tier{b}_rows", torch.zeros(n, dtype=torch.int32))
            layer.register_buffer(f"tier{b}_packed", torch.zeros(n, _packed_cols(in_features, b), dtype=torch.uint8))
            layer.register_buffer(f"tier{b}_scales", torch.ones(n, g, dtype=torch.float32))
            layer.register_buffer(f"tier{b}_zp", torch.zeros(n, g, dtype=torch.int32))
            layer.tier_bits.append(b)
        return layer

    # ── tensor-parallel shards ──────────────────────────────────────────────
    def tp_shard(self, dim: str, rank: int, world: int) -> "CSAQLinear":
        """The rank's part of this layer for tensor parallelism, as a mixed-row
        layer. ``dim="col"``: output rows [rank*N/world, (rank+1)*N/world);
        ``dim="row"``: input columns [rank*K/world, ...), which must be a
        multiple of 128 wide so quantisation groups stay whole (the bias then
        stays on rank 0 only, because the partial outputs are summed).
        Protected rows and their fp16 copies are split the same way."""
        N, K = self.out_features, self.in_features
        if dim not in ("col", "row"):
            raise ValueError("dim must be 'col' or 'row'")
        full = N if dim == "col" else K
        if full % world:
            raise ValueError(f"{full} does not split over {world} ranks")
        lo, hi = rank * full // world, (rank + 1) * full // world
        if dim == "row" and (lo % 128 or hi % 128):
            raise ValueError("row shards must be 128-column aligned")
        hi_rows = getattr(self, "_csaq_hi_rows", None)
        bk = getattr(self, "_csaq_fp16_backup", None)
        bias = self.bias
        # the tiers as stored (on the buffers' own device), protected rows last in each
        src = []
        if self.tier_bits:
            for b in self.tier_bits:
                sc = getattr(self, f"tier{b}_scales")
                src.append((b, getattr(self, f"tier{b}_rows").long(), getattr(self, f"tier{b}_packed"),
                            sc.reshape(sc.shape[0], -1), getattr(self, f"tier{b}_zp").reshape(sc.shape[0], -1)))
        else:
            b = self.bits
            rows = torch.arange(N, device=self.weight_packed.device)
            codes = self.weight_packed.reshape(N, -1)
            sc, zp = self.weight_scales.reshape(N, -1).float(), self.weight_zp.reshape(N, -1)
            if hi_rows is not None and hi_rows.numel():
                prot = torch.zeros(N, dtype=torch.bool, device=rows.device)
                prot[hi_rows.to(rows.device)] = True
                order = torch.cat([rows[~prot], rows[prot]])
                rows, codes, sc, zp = order, codes[order], sc[order], zp[order]
            src.append((b, rows, codes, sc, zp))
        parts = []
        for b, rows, codes, sc, zp in src:
            if dim == "col":
                keep = (rows >= lo) & (rows < hi)
                rows, codes, sc, zp = rows[keep] - lo, codes[keep], sc[keep], zp[keep]
            else:
                b0, b1 = (lo * b) // 8, (hi * b) // 8
                codes = codes[:, b0:b1]
                if b != 16 and sc.shape[-1] > 1:
                    gs = K // sc.shape[-1] if self.group_size <= 0 else self.group_size
                    g0, g1 = lo // gs, hi // gs
                    sc, zp = sc[:, g0:g1], zp[:, g0:g1]
            if rows.numel():
                parts.append((b, rows, codes, sc, zp.to(torch.int32)))
        n_out, n_in = (hi - lo, K) if dim == "col" else (N, hi - lo)
        if dim == "col":
            b_sh = None if bias is None else bias[lo:hi]
        else:
            b_sh = bias if rank == 0 else None
        grouped = self.tier_bits and 0 < self.group_size < K or (not self.tier_bits and self.weight_scales.dim() == 2)
        counts = {b: r.numel() for b, r, *_ in parts}
        out = CSAQLinear(n_in, n_out, max(counts, key=counts.__getitem__), bias=b_sh,
                         group_size=self.group_size if grouped else -1)
        dev = parts[0][2].device
        out.weight_packed = torch.zeros(0, dtype=torch.uint8, device=dev)
        out.weight_scales = torch.zeros(0, dtype=torch.float32, device=dev)
        out.weight_zp = torch.zeros(0, dtype=torch.int32, device=dev)
        for b, rows, codes, sc, zp in parts:
            out.register_buffer(f"tier{b}_rows", rows.to(torch.int32).contiguous())
            out.register_buffer(f"tier{b}_packed", codes.contiguous())
            out.register_buffer(f"tier{b}_scales", sc.reshape(rows.numel(), -1).contiguous())
            out.register_buffer(f"tier{b}_zp", zp.reshape(rows.numel(), -1).contiguous())
            out.tier_bits.append(b)
        if hi_rows is not None and hi_rows.numel():
            if dim == "col":
                keep = (hi_rows >= lo) & (hi_rows < hi)
                out.set_protected_rows(hi_rows[keep] - lo, bk[keep])
            else:
                out.set_protected_rows(hi_rows, bk[:, lo:hi])
        return out

    # ── verify-pass protection (apply_csaq, csaq/core.py:393-407) ───────────
    def set_protected_rows(self, hi_rows: torch.Tensor, fp16_backup: torch.Tensor) -> None:
        """Register the protected rows and their fp16 weights.

        The reference stores the fp16 cast of the *dequantised* rows
        (csaq/core.py:401-402), which makes the verify pass identical to the
        draft pass; this build stores the fp16 of the original weights.
        """
        dev = self._buf_device()
        hi = torch.sort(hi_rows.to(torch.int64)).values
        self.register_buffer("_csaq_hi_rows", hi.to(dev), persistent=False)
        self.register_buffer("_csaq_fp16_backup", fp16_backup.to(torch.float16).contiguous().to(dev),
                             persistent=False)
        self._gemv_cache = {}

    def _buf_device(self) -> torch.device:
        return self.weight_scales.device

    # ── GEMV descriptors ──────────────────────────────────────────────────────
    def _gpu(self, t: torch.Tensor) -> torch.Tensor:
        return _on_gpu(t)

    def _tiers(self) -> List[_Tier]:
        K = self.in_features
        hi = getattr(self, "_csaq_hi_rows", None)
        prot = None
        if hi is not None and hi.numel():
            prot = torch.zeros(self.out_features, dtype=torch.bool, device=hi.device)
            prot[hi] = True
        tiers: List[_Tier] = []
        if self.tier_bits:
            for b in self.tier_bits:
                rows = self._gpu(getattr(self, f"tier{b}_rows"))
                n = rows.numel()
                if n == 0:
                    continue
                n_ver = n - (int(prot.to(rows.device)[rows.long()].sum()) if prot is not None else 0)
                s = self._gpu(getattr(self, f"tier{b}_scales")).contiguous()
                z = _zps_u8(self._gpu(getattr(self, f"tier{b}_zp")))
                gs = self.group_size if (b != 16 and 0 < self.group_size < K) else K
                tiers.append(_Tier(b, rows, self._gpu(getattr(self, f"tier{b}_packed")).contiguous(),
                                   s, z, gs, s.shape[-1] if s.dim() == 2 else 1, n_ver))
            return tiers
        # uniform reference layer: one tier in natural row order; with
        # protected rows the tier is re-ordered (unprotected first)
        b = self.bits
        rows = torch.arange(self.out_features, dtype=torch.int32, device=self._gpu(self.weight_scales).device)
        codes = self._gpu(self.weight_packed)
        s = self._gpu(self.weight_scales).float()
        z = self._gpu(self.weight_zp)
        if b == 16:
            codes = codes.reshape(self.out_features, 2 * K)
        s = s.reshape(self.out_features, -1)
        z = z.reshape(self.out_features, -1)
        G = s.shape[1]
        gs = K if G == 1 else (self.group_size if self.group_size > 0 else (K + G - 1) // G)
        n_ver = self.out_features
        if prot is not None:
            order = torch.cat([torch.nonzero(~prot).flatten(), torch.nonzero(prot).flatten()]).to(codes.device)
            rows = order.to(torch.int32)
            codes, s, z = codes[order], s[order], z[order]
            n_ver = int((~prot).sum())
        tiers.append(_Tier(b, rows.contiguous(), codes.contiguous(), s.contiguous(), _zps_u8(z), gs, G,
                           n_ver))
        return tiers

    def _blocks_for(self, bits: int, n_rows: int, codes: torch.Tensor, scales, zps_u8, group_size,
                    n_groups) -> Optional[torch.Tensor]:
        """GEMV block layout of one tier (csaq_repack_tiles), or None when the
        shape is served by the CUDA-core kernel only."""
        K = self.in_features
        if K % 128 != 0 or (bits != 16 and group_size % 128 != 0):
            return None
        nbytes = lib().csaq_tile_blocks_bytes(bits, n_rows, K)
        blocks = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=codes.device)
        d = CsaqTier(bits=bits, n_rows=n_rows, group_size=group_size, n_groups=n_groups,
                     row_bytes=codes.shape[1], codes=codes.data_ptr(),
                     scales=ptr(scales), zps=ptr(zps_u8))
        check(lib().csaq_repack_tiles(ctypes.byref(d), K, blocks.data_ptr(), stream_of(codes)),
              "repack_tiles")
        return blocks

    def _descriptors(self, verify: bool):
        key = ("verify" if verify else "draft", )
        ent = self._gemv_cache.get(key)
        if ent is not None:
            return ent
        K = self.in_features
        tiers = self._gemv_cache.get("tiers")
        if tiers is None:
            tiers = self._tiers()
            for t in tiers:
                t_blocks = self._blocks_for(t.bits, t.rows.numel(), t.codes, t.scales, t.zps_u8,
                                            t.group_size, t.n_groups)
                self._gemv_cache[("blocks", t.bits)] = t_blocks
            self._gemv_cache["tiers"] = tiers
        descs, keep = [], [tiers]
        for t in tiers:
            n = t.n_verify if verify else t.rows.numel()
            if n == 0:
                continue
            blk = self._gemv_cache[("blocks", t.bits)]
            keep.append(blk)
            descs.append(CsaqTier(bits=t.bits, n_rows=n, group_size=t.group_size, n_groups=t.n_groups,
                                  row_bytes=t.codes.shape[1], codes=t.codes.data_ptr(),
                                  scales=t.scales.data_ptr(), zps=t.zps_u8.data_ptr(),
                                  out_rows=t.rows.data_ptr(), blocks=ptr(blk), y=None,
                                  ldy=self.out_features, bias=None, residual=None, ldr=0))
        if verify and getattr(self, "_csaq_hi_rows", None) is not None and self._csaq_hi_rows.numel():
            hi = self._gpu(self._csaq_hi_rows).to(torch.int32).contiguous()
            bk = self._gpu(self._csaq_fp16_backup).contiguous().view(torch.uint8)
            one = torch.ones(1, dtype=torch.float32, device=bk.device)
            zero = torch.zeros(1, dtype=torch.uint8, device=bk.device)
            blk = self._blocks_for(16, hi.numel(), bk, None, None, K, 1)
            keep += [hi, bk, one, zero, blk]
            descs.append(CsaqTier(bits=16, n_rows=hi.numel(), group_size=K, n_groups=1,
                                  row_bytes=bk.shape[1], codes=bk.data_ptr(), scales=one.data_ptr(),
                                  zps=zero.data_ptr(), out_rows=hi.data_ptr(), blocks=ptr(blk),
                                  y=None, ldy=self.out_features, bias=None, residual=None, ldr=0))
        ent = (descs, keep)
        self._gemv_cache[key] = ent
        return ent

    def _bias_as(self, dtype: torch.dtype, device) -> Optional[torch.Tensor]:
        if self.bias is None:
            return None
        key = ("bias", dtype)
        b = self._gemv_cache.get(key)
        if b is None or b.device != device:
            b = self.bias.detach().to(device=device, dtype=dtype).contiguous()
            self._gemv_cache[key] = b
        return b

    def gemv_descriptors(self, y: torch.Tensor, verify: bool = False,
                         residual: Optional[torch.Tensor] = None) -> List[CsaqTier]:
        """ctypes tier descriptors writing into ``y`` (M x ldy); used to fuse
        several linears that read the same input into one launch."""
        descs, _ = self._descriptors(verify)
        bias = self._bias_as(y.dtype, y.device)
        out = []
        for d in descs:
            e = CsaqTier()
            ctypes_copy(e, d)
            e.y = y.data_ptr()
            e.ldy = y.stride(0)
            e.bias = ptr(bias)
            if residual is not None:
                e.residual = residual.data_ptr()
                e.ldr = residual.stride(0)
            out.append(e)
        return out

    def _get_weight_fp32(self) -> torch.Tensor:
        """Dequantised fp32 weight (csaq/kernels.py:450-468)."""
        N, K = self.out_features, self.in_features
        if self.tier_bits:
            W = torch.empty(N, K, dtype=torch.float32, device=self._gpu(self.weight_scales).device)
            for t in self._tiers():
                if t.bits == 16:
                    w = _dequant_raw(t.codes, None, None, 16, t.rows.numel(), K, -1)
                else:
                    w = _dequant_raw(t.codes, t.scales, getattr(self, f"tier{t.bits}_zp"), t.bits,
                                     t.rows.numel(), K, t.group_size if t.group_size < K else -1,
                                     nan_to_num=True)
                W[t.rows.long()] = w
            return W.to(self._buf_device())
        if self.bits == 16:
            return _dequant_raw(self.weight_packed, None, None, 16, N, K, -1).to(self._buf_device())
        gs = -1 if self.weight_scales.dim() == 1 else self.group_size
        return _dequant_raw(self.weight_packed, self.weight_scales, self.weight_zp, self.bits, N, K,
                            gs, nan_to_num=True).to(self._buf_device())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        K, N = self.in_features, self.out_features
        dev = x.device
        xg = _on_gpu(x)
        x2 = xg.reshape(-1, K)
        if x2.stride(1) != 1 or x2.stride(0) != K:
            x2 = x2.contiguous()
        M = x2.shape[0]
        y = torch.empty(M, N, dtype=x2.dtype, device=x2.device)
        if M:
            descs = self.gemv_descriptors(y, verify=self.verify_mode)
            if M >= GEMM_MIN_TOKENS and K % 64 == 0 and x2.dtype in (torch.float16, torch.bfloat16):
                _lib.qgemm(descs, K, x2, M)   # many tokens: the tensor-core GEMM
            else:
                _lib.qgemv(descs, K, x2, M)
        y = y.view(*x.shape[:-1], N)
        return y if y.device == dev else y.to(dev)

    def extra_repr(self) -> str:
        if self.tier_bits:
            return (f"in={self.in_features}, out={self.out_features}, tiers={self.tier_bits}, "
                    f"group_size={self.group_size}")
        return (f"in={self.in_features}, out={self.out_features}, bits={self.bits}, "
                f"group_size={self.group_size}")


def ctypes_copy(dst: CsaqTier, src: CsaqTier) -> None:
    import ctypes
    ctypes.pointer(dst)[0] = src


def _get_submodule(model: nn.Module, name: str) -> Optional[nn.Module]:
    mod: nn.Module = model
    for part in name.split("."):
        child = getattr(mod, part, None)
        if child is None:
            return None
        mod = child
    return mod
