"""Failure detection of the tensor-parallel exchange (csaq_tp_exchange_sum),
on one GPU and without a fault.

The exchange kernel signals its peers and then waits, bounded, for their
signals. Here the "peer" of rank 0 is a second local buffer and flag array
that nothing ever writes, and the wait limit is set low (csaq_p2p_set_spin_limit):
the wait must run out, the kernel must still finish (its sum uses whatever
the peer buffer holds), the host must read the abandoned wait from
csaq_p2p_errors, the CUDA context must stay usable, and a broken group must
not wait again. No peer memory, multicast or second process is involved.
"""

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _exchange(G, out, N, M):
    from csaq._lib import check, lib, stream_of
    check(lib().csaq_tp_exchange_sum(ctypes.byref(G), 0, N, out.data_ptr(), N, M, N, 2, stream_of(out)),
          "tp_exchange")


def test_tp_exchange_wait_runs_out_and_returns():
    from csaq import _lib
    from csaq._lib import check, lib
    M, N = 1, 256  # one CTA: each CTA of the exchange waits (and gives up) on its own
    g = torch.Generator().manual_seed(3)
    parts = [torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV) for _ in range(2)]
    flags = [torch.zeros(2, dtype=torch.int64, device=DEV) for _ in range(2)]  # flags[0][1]: never written
    seq = torch.zeros(1, dtype=torch.int64, device=DEV)
    ticket = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV)
    before = out.clone()
    G = _lib.CsaqP2PGroup(n_ranks=2, rank=0)
    for r in range(2):
        G.parts[r] = parts[r].data_ptr()
        G.flags[r] = flags[r].data_ptr()
    G.seq, G.ticket, G.err = seq.data_ptr(), ticket.data_ptr(), err.data_ptr()
    check(lib().csaq_p2p_set_spin_limit(4096), "spin_limit")
    try:
        t0 = time.time()
        _exchange(G, out, N, M)
        torch.cuda.synchronize()
        elapsed = time.time() - t0
    finally:
        check(lib().csaq_p2p_set_spin_limit(1 << 22), "spin_limit")
    assert elapsed < 5.0
    n = ctypes.c_int64(-1)
    check(lib().csaq_p2p_errors(ctypes.byref(G), ctypes.byref(n)), "p2p_errors")
    assert n.value == 1
    # it signalled the peer (rank 1's array, slot 0) and advanced its exchange count
    assert int(flags[1][0]) == 1 and int(seq) == 1 and int(ticket) == 0
    # and still wrote out + part_0 + part_1 in rank order (fp32, rounded once)
    exp = ((before.float() + parts[0].float()) + parts[1].float()).to(torch.bfloat16)
    assert torch.equal(out, exp)
    # the context is usable
    assert float(torch.ones(8, device=DEV).sum()) == 8.0
    # a broken group does not wait again: the next exchange returns at once, the count stays 1
    t0 = time.time()
    _exchange(G, out, N, M)
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    check(lib().csaq_p2p_errors(ctypes.byref(G), ctypes.byref(n)), "p2p_errors")
    assert n.value == 1 and int(seq) == 2


def test_spin_limit_argument_checked():
    from csaq._lib import lib
    assert lib().csaq_p2p_set_spin_limit(0) == -1
