"""Tensor-parallel decode runtime on 2 GPUs (skipped with fewer).

Two NCCL ranks run a quantised tiny Llama through DecodeRuntime with a TP
group: the prefill logits match the single-GPU runtime's within 3e-2 (the
partial sums are added in a different order), and greedy self-speculative
output equals greedy decoding with the verify weights under TP. The combine
after the row-split projections goes through peer memory (csaq_tp_exchange_sum,
no abandoned waits) and gives bitwise the results of the NCCL all-gather path.
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _np(obj):
    """Tensors -> numpy arrays, recursively: a tensor on a multiprocessing queue
    is a shared-memory handle that dies with the worker process."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().float().cpu().numpy() if obj.is_floating_point() else obj.detach().cpu().numpy()
    if isinstance(obj, dict):
        return {k: _np(v) for k, v in obj.items()}
    return obj


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build(dev):
    from csaq import _synthetic as syn
    from csaq.config import CSAQConfig
    from csaq.core import apply_csaq, solve_clique_budget
    model = syn.build_decoder("tiny-llama", device=dev, seed=4, dtype=torch.bfloat16)
    sal = syn.synthetic_salience(model, seed=5)
    cfg = CSAQConfig(target_bits=4.0, bit_options=[4, 8, 16], group_size=128, protection_floor=0.10,
                     clique_mode="per_channel")
    cliques = {n: [[i] for i in range(s.shape[0])] for n, s in sal.items()}
    budget, _, _ = solve_clique_budget(sal, cliques, cfg)
    cmap = apply_csaq(model, budget, sal, cfg, verbose=False)
    return model, cmap


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    out = {}
    try:
        from csaq.runtime import DecodeRuntime
        model, _ = _build(dev)
        prompt = torch.randint(0, 2048, (1, 40), generator=torch.Generator().manual_seed(6)).to(dev)
        rt = DecodeRuntime(model, 1, 256, 4, tp_group=dist.group.WORLD)
        out["peer_memory"] = rt.p2p is not None
        rt.reset(prompt, 24, verify=True)
        out["tp_logits"] = rt.prefill_logits.float().cpu()
        rt.generate_greedy(24, verify=True)
        greedy = rt.outputs().cpu()
        rt.reset(prompt, 24, verify=True)
        rt.generate_speculative(24)
        out["spec_equals_greedy"] = torch.equal(rt.outputs().cpu()[:, :24], greedy[:, :24])
        out["p2p_errors"] = rt.p2p.errors() if rt.p2p is not None else -1
        rt.release()
        del rt
        # the NCCL all-gather combine adds the same partials in the same order
        os.environ["CSAQ_TP_EXCHANGE"] = "nccl"
        rt2 = DecodeRuntime(model, 1, 256, 4, tp_group=dist.group.WORLD)
        rt2.reset(prompt, 24, verify=True)
        out["nccl_logits_equal"] = torch.equal(rt2.prefill_logits.float().cpu(), out["tp_logits"])
        rt2.generate_greedy(24, verify=True)
        out["nccl_greedy_equal"] = torch.equal(rt2.outputs().cpu()[:, :24], greedy[:, :24])
        rt2.release()
        del rt2
        os.environ.pop("CSAQ_TP_EXCHANGE")
        torch.cuda.synchronize()
        if rank == 0:
            one = DecodeRuntime(model, 1, 256, 4)
            one.reset(prompt, 8, verify=True)
            out["tp1_logits"] = one.prefill_logits.float().cpu()
        dist.barrier()
        q.put((rank, _np(out)))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_runtime_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        assert res[r]["spec_equals_greedy"], r
        assert res[r]["peer_memory"], r
        assert res[r]["p2p_errors"] == 0, r
        assert res[r]["nccl_logits_equal"] and res[r]["nccl_greedy_equal"], r
    a, b = torch.from_numpy(res[0]["tp_logits"]), torch.from_numpy(res[0]["tp1_logits"])
    assert torch.equal(torch.from_numpy(res[0]["tp_logits"]), torch.from_numpy(res[1]["tp_logits"]))
    err = float((a - b).norm() / b.norm())
    cos = float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0))
    assert err < 3e-2 and cos > 0.999, (err, cos)


def _dp_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        from csaq import _synthetic as syn
        from csaq.config import CSAQConfig
        from csaq.core import CausalProfiler
        model = syn.build_decoder("tiny-llama", device=dev, seed=0, dtype=torch.float32)
        g = torch.Generator().manual_seed(3)
        calib = [{"input_ids": torch.randint(0, 2048, (1, 32), generator=g)} for _ in range(4)]
        cfg = CSAQConfig(clique_threshold=0.6, salience_alpha=1.0)
        sal, cl = CausalProfiler(model, cfg, dp_group=dist.group.WORLD).profile(calib, verbose=False)
        out = {"sal": {k: v.cpu() for k, v in sal.items()}, "cl": cl}
        dist.barrier()
        if rank == 0:
            model.zero_grad()
            sal1, cl1 = CausalProfiler(model, cfg).profile(calib, verbose=False)
            out["sal1"] = {k: v.cpu() for k, v in sal1.items()}
            out["cl1"] = cl1
        q.put((rank, _np(out)))
    finally:
        dist.destroy_process_group()


def test_data_parallel_calibration_two_gpus():
    """Two ranks profiling batches 0,2 and 1,3 give the single-GPU salience
    (within 1e-3) and exactly the single-GPU cliques (integer count sums)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    r0, r1 = res[0], res[1]
    assert r0["cl"] == r1["cl"] == r0["cl1"]
    for k, v in r0["sal1"].items():
        a, b, one = torch.from_numpy(r0["sal"][k]), torch.from_numpy(r1["sal"][k]), torch.from_numpy(v)
        assert torch.equal(a, b), k
        assert torch.allclose(a, one, rtol=1e-3, atol=1e-12), k


def _rowq_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        from csaq.kernels import quantize_per_channel
        W = (torch.randn(1000, 1024, generator=torch.Generator().manual_seed(8)) * 0.02).to(torch.bfloat16).to(dev)
        W[torch.arange(0, 1000, 97)] *= 10.0
        out = {}
        n = W.shape[0] // world
        for bits in (2, 4, 8):
            for gs in (128, -1):
                mine = quantize_per_channel(W[rank * n:(rank + 1) * n], bits, gs)
                parts = {}
                for name, t in (("q", mine.qdata), ("s", mine.scales), ("z", mine.zero_points)):
                    t = t.contiguous().to(dev)
                    gathered = [torch.empty_like(t) for _ in range(world)]
                    dist.all_gather(gathered, t)
                    parts[name] = torch.cat(gathered)
                full = quantize_per_channel(W, bits, gs)
                out[(bits, gs)] = all(torch.equal(parts[k], v.to(dev)) for k, v in
                                      (("q", full.qdata), ("s", full.scales), ("z", full.zero_points)))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_row_parallel_quantisation_two_gpus():
    """Rows quantise independently (csaq/kernels.py:77-158): two ranks
    quantising their halves of the rows and all-gathering codes, scales and
    zero points reproduce the one-GPU quantisation bit for bit, with no other
    exchange."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rowq_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        assert all(res[r].values()), res[r]
