"""Host logic of the multi-GPU key-range split (fa_b200.kvsplit) on two CPU
ranks over gloo.  The GPU kernels are replaced by numpy stand-ins with the same
contract (partial over a key range with global causal positions; LSE merge),
so what is tested is the zig-zag chunking, the all-to-all exchange layout and
the final merge; the result is compared with the oracle of the whole slice."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fa_b200.kvsplit import row_blocks, zigzag_chunks


def _partial_np(q, k, v, out, lse, causal, q_offset, k_offset):
    qn, kn, vn = q[0].numpy().astype(np.float64), k[0].numpy().astype(np.float64), v[0].numpy().astype(np.float64)
    s = qn @ kn.T / np.sqrt(qn.shape[1])
    if causal:
        qi = q_offset + np.arange(qn.shape[0])[:, None]
        kj = k_offset + np.arange(kn.shape[0])[None, :]
        s = np.where(kj <= qi, s, -np.inf)
    m = s.max(1, keepdims=True)
    ok = np.isfinite(m[:, 0])
    p = np.where(ok[:, None], np.exp(s - np.where(ok[:, None], m, 0)), 0.0)
    l = p.sum(1)
    o = np.where(ok[:, None], (p @ vn) / np.where(l > 0, l, 1)[:, None], 0.0)
    out[0].copy_(torch.from_numpy(o.astype(np.float32)))
    lse[0].copy_(torch.from_numpy(np.where(ok, m[:, 0] + np.log(np.where(l > 0, l, 1)), -np.inf).astype(np.float32)))


def _combine_np(o_parts, lse_parts, out, lse_out):
    lp = lse_parts.numpy().astype(np.float64)
    M = lp.max(0)
    fin = np.isfinite(M)
    w = np.where(fin[None, :], np.exp(lp - np.where(fin, M, 0)[None, :]), 0.0)
    L = w.sum(0)
    o = (w[:, :, None] * o_parts.numpy()).sum(0) / np.where(L > 0, L, 1)[:, None]
    out.copy_(torch.from_numpy(o.astype(np.float32)))
    lse_out.copy_(torch.from_numpy(np.where(L > 0, M + np.log(np.where(L > 0, L, 1)), -np.inf).astype(np.float32)))


def _worker(rank, world, port, rows, d, causal, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fa_b200.kvsplit import kv_split_forward
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, rows, d, generator=g)
    k = torch.randn(1, rows, d, generator=g)
    v = torch.randn(1, rows, d, generator=g)
    out, lse, (a, b) = kv_split_forward(q, k, v, causal, partial_fn=_partial_np,
                                        combine_fn=_combine_np)
    ret[rank] = (a, b, out.numpy().copy(), lse.numpy().copy())
    dist.destroy_process_group()


def test_zigzag_chunks_cover_keys_once():
    for seq, world in ((131072, 8), (1000, 2), (7, 4)):
        seen = []
        for r in range(world):
            for c in zigzag_chunks(seq, world, r):
                seen.extend(range(c.start, c.stop))
        assert sorted(seen) == list(range(seq))
    with pytest.raises(ValueError):
        row_blocks(10, 4)


@pytest.mark.parametrize("causal", [True, False])
def test_kv_split_two_gloo_ranks_matches_oracle(causal):
    import oracle as O
    world, rows, d = 2, 96, 16
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ret = mp.Manager().dict()
    mp.spawn(_worker, args=(world, port, rows, d, causal, ret), nprocs=world, join=True)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, rows, d, generator=g)
    k = torch.randn(1, rows, d, generator=g)
    v = torch.randn(1, rows, d, generator=g)
    want, wlse = O.flash_v2(q.numpy().ravel(), k.numpy().ravel(), v.numpy().ravel(), rows, rows,
                            d, causal)
    want = want.reshape(rows, d)
    for r in range(world):
        a, b, out, lse = ret[r]
        assert np.max(np.abs(out - want[a:b])) < 1e-5
        assert np.max(np.abs(lse - wlse[a:b])) < 1e-5
