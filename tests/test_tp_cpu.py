"""Tensor-parallel sharding of CSAQLinear, on CPU ranks over gloo.

Two processes shard the same synthetic mixed-tier layer (fp16 / 8-bit /
4-bit rows, group 128, with protected rows) by output rows ("col") and by
128-aligned input columns ("row"), compute their partial outputs with the
oracle's dequantise-then-matmul, all-gather them, and recombine: the column
shards concatenate to the full layer's output exactly, and the row shards
summed in rank order match it within float tolerance. The protected rows and
their fp16 copies must be split consistently. No GPU is used.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(uniform: bool):
    from csaq.kernels import CSAQLinear
    g = torch.Generator().manual_seed(3)
    N, K = 96, 512
    if uniform:
        layer = CSAQLinear(K, N, 4, group_size=128)
        layer.weight_packed.copy_(torch.randint(0, 256, layer.weight_packed.shape, generator=g,
                                                dtype=torch.int32).to(torch.uint8))
        layer.weight_scales.copy_(torch.rand(layer.weight_scales.shape, generator=g) * 0.01)
        layer.weight_zp.copy_(torch.randint(0, 16, layer.weight_zp.shape, generator=g, dtype=torch.int32))
    else:
        layer = CSAQLinear.empty_tiers(K, N, {16: 16, 8: 32, 4: 48}, group_size=128)
        perm = torch.randperm(N, generator=g).to(torch.int32)
        start = 0
        for b in layer.tier_bits:
            n = getattr(layer, f"tier{b}_rows").numel()
            getattr(layer, f"tier{b}_rows").copy_(torch.sort(perm[start:start + n]).values)
            start += n
            pk = getattr(layer, f"tier{b}_packed")
            if b == 16:
                pk.copy_((torch.randn(n, K, generator=g) * 0.02).to(torch.float16).view(torch.uint8))
            else:
                pk.copy_(torch.randint(0, 256, pk.shape, generator=g, dtype=torch.int32).to(torch.uint8))
                getattr(layer, f"tier{b}_scales").copy_(torch.rand(n, K // 128, generator=g) * 0.01)
                getattr(layer, f"tier{b}_zp").copy_(torch.randint(0, 2 ** b - 1, (n, K // 128), generator=g,
                                                                  dtype=torch.int32))
    hi = torch.tensor([1, 7, 40, 41, 90])
    layer.set_protected_rows(hi, (torch.randn(5, K, generator=g) * 0.02).to(torch.float16))
    return layer


def _dense(layer) -> np.ndarray:
    """The layer's dequantised weight, with the oracle."""
    from oracle import csaq_oracle as O
    N, K = layer.out_features, layer.in_features
    W = np.zeros((N, K), np.float32)
    if layer.tier_bits:
        for b in layer.tier_bits:
            rows = getattr(layer, f"tier{b}_rows").long().numpy()
            codes = getattr(layer, f"tier{b}_packed").numpy()
            if b == 16:
                W[rows] = codes.view(np.float16).astype(np.float32).reshape(rows.size, K)
            else:
                W[rows] = O.dequantize_grouped(codes, getattr(layer, f"tier{b}_scales").numpy(),
                                               getattr(layer, f"tier{b}_zp").numpy(), b, rows.size, K, 128)
    else:
        W[:] = O.dequantize_grouped(layer.weight_packed.numpy(), layer.weight_scales.numpy(),
                                    layer.weight_zp.numpy(), layer.bits, N, K, layer.group_size)
    return W


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        x = torch.randn(3, 512, generator=torch.Generator().manual_seed(9))
        for uniform in (False, True):
            full = _layer(uniform)
            Wf = torch.from_numpy(_dense(full))
            for dim in ("col", "row"):
                sh = full.tp_shard(dim, rank, world)
                Ws = torch.from_numpy(_dense(sh))
                if dim == "col":
                    part = x @ Ws.T                                   # (3, N/world)
                    gathered = [torch.zeros_like(part) for _ in range(world)]
                    dist.all_gather(gathered, part)
                    y = torch.cat(gathered, dim=1)
                else:
                    k0 = rank * 512 // world
                    part = x[:, k0:k0 + 512 // world] @ Ws.T          # (3, N) partial sum
                    gathered = [torch.zeros_like(part) for _ in range(world)]
                    dist.all_gather(gathered, part)
                    y = gathered[0]
                    for p in gathered[1:]:
                        y = y + p
                ref = x @ Wf.T
                out[(uniform, dim, "exact" if dim == "col" else "close")] = (
                    torch.equal(y, ref) if dim == "col" else bool(torch.allclose(y, ref, rtol=1e-5, atol=1e-5)))
                # protected rows: the shard's fp16 copies are the matching slice of the full layer's
                hi_f, bk_f = full._csaq_hi_rows, full._csaq_fp16_backup
                if dim == "col":
                    lo = rank * full.out_features // world
                    keep = (hi_f >= lo) & (hi_f < lo + full.out_features // world)
                    ok = torch.equal(sh._csaq_hi_rows, hi_f[keep] - lo) and torch.equal(sh._csaq_fp16_backup, bk_f[keep])
                else:
                    k0 = rank * 512 // world
                    ok = torch.equal(sh._csaq_hi_rows, hi_f) and torch.equal(sh._csaq_fp16_backup,
                                                                             bk_f[:, k0:k0 + 512 // world])
                out[(uniform, dim, "protected")] = bool(ok)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_tp_shards_recombine_over_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out in results:
        for key, ok in out.items():
            assert ok, (rank, key)


def test_tp_shard_rejects_bad_splits():
    full = _layer(False)
    with pytest.raises(ValueError):
        full.tp_shard("row", 0, 3)   # 512 / 3 is not whole
    with pytest.raises(ValueError):
        full.tp_shard("row", 0, 8)   # 64-column shards break the 128-column groups
    with pytest.raises(ValueError):
        full.tp_shard("diag", 0, 2)
