"""Row-sharded linear (spectra_b200.sharded) on CPU: 2, 4 and 8 gloo ranks, each
computing its rows with the oracle, must assemble exactly the oracle's
full-layer output (M = 1 and M > 1, ragged and empty last shards, outliers,
bias), and the sharded greedy head must pick the oracle's argmax."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spectra_b200.sharded import ShardedW4A16Linear, shard_bounds


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_local(x2d, packed, scales, zeros, idx, ow, bias, marlin, out=None):
    """One rank's slice by the oracle (the reference's routing: GEMV with bias at
    M = 1, GEMM then + bias otherwise), rounded to x's dtype; written into
    ``out`` when given (the module's local_fn contract)."""
    y = _oracle_slice(x2d, packed, scales, zeros, idx, ow, bias, marlin)
    if out is not None:
        out.copy_(y)
    return y


def _oracle_argmax(y, offset):
    from oracle import ops as P
    yn = y.float().numpy()
    i = P.argmax(yn)
    return torch.from_numpy(yn[np.arange(len(i)), i]), torch.from_numpy(i + offset)


def _oracle_slice(x2d, packed, scales, zeros, idx, ow, bias, marlin):
    from oracle import w4a16 as O
    xn = x2d.float().numpy().astype(np.float16)
    p, s, z = packed.numpy(), scales.numpy(), zeros.numpy()
    has = idx is not None and idx.numel() > 0
    own = ow.float().numpy().astype(np.float16) if has else None
    if x2d.shape[0] == 1:
        b = bias.float().numpy().astype(np.float16) if bias is not None else None
        _, y, _ = O.gemv(xn, "f16", p, s, z, bias=b, bias_dtype="f16" if b is not None else None,
                         outlier_idx=idx.numpy() if has else None, outlier_w=own, ow_dtype="f16", marlin=marlin)
        return torch.from_numpy(np.asarray(y, np.float64).reshape(1, -1)).to(torch.float16)
    _, c, _ = O.gemm(xn, "f16", p, s, z, outlier_idx=idx.numpy() if has else None, outlier_w=own,
                     ow_dtype="f16", marlin=marlin)
    y = torch.from_numpy(np.asarray(c, np.float64)).to(torch.float16)
    return y + bias if bias is not None else y


def _layer(N, K, n_out, seed):
    from tests.helpers import random_format
    f = random_format(N, K, n_out, seed=seed, ow_dtype="f16")
    g = torch.Generator().manual_seed(seed)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.float16)
    return (torch.from_numpy(f["packed"]), torch.from_numpy(f["scales"]), torch.from_numpy(f["zeros"]),
            torch.from_numpy(f["outlier_idx"]), f["outlier_w_t"], bias)


def _worker(rank, world, port, cases, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = []
        for N, K, n_out, M, seed in cases:
            p, s, z, idx, ow, bias = _layer(N, K, n_out, seed)
            lin = ShardedW4A16Linear(p, s, z, outlier_idx=idx, outlier_w=ow, bias=bias, marlin_layout=True,
                                     device=torch.device("cpu"), local_fn=_oracle_local, argmax_fn=_oracle_argmax)
            x = (torch.randn(M, K, generator=torch.Generator().manual_seed(seed + 1))).to(torch.float16)
            y = lin(x)
            y2 = lin(x)  # the persistent slice buffer is reused
            assert torch.equal(y, y2)
            res.append((y.numpy(), lin.greedy(x).numpy()))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


CASES = [(256, 128, 4, 1, 1), (250, 128, 4, 1, 2), (250, 256, 0, 3, 3), (97, 64, 5, 2, 4)]
# 4 and 8 ranks: ragged shards (1003 = 8 x 126 - 5), a shard count that leaves
# the last ranks empty (9 rows over 8 ranks: 2,2,2,2,1,0,0,0), and a vocabulary-
# shaped head (N = 1000 ~ 128256 / 128) at M = 1 and M > 1
CASES_WIDE = [(1003, 128, 3, 1, 5), (9, 64, 2, 1, 6), (9, 64, 2, 3, 7), (1000, 256, 6, 1, 8), (1003, 128, 0, 4, 9)]


def test_shard_bounds_cover_rows_once():
    for N in (1, 7, 250, 256):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                ns, lo, hi = shard_bounds(N, world, r)
                assert ns == -(-N // world) and 0 <= hi - lo <= ns
                rows.extend(range(lo, hi))
            assert rows == list(range(N))
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _run_world(world, cases):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for ci, (N, K, n_out, M, seed) in enumerate(cases):
        p, s, z, idx, ow, bias = _layer(N, K, n_out, seed)
        x = (torch.randn(M, K, generator=torch.Generator().manual_seed(seed + 1))).to(torch.float16)
        full = _oracle_local(x, p, s, z, idx if n_out else None, ow if n_out else None, bias, True).numpy()
        from oracle import ops as P
        want_tok = P.argmax(full.astype(np.float32))
        for r in range(world):
            y, tok = got[r][ci]
            assert y.shape == (M, N)
            np.testing.assert_array_equal(y, full, err_msg=f"case {ci} rank {r}")
            np.testing.assert_array_equal(tok, want_tok, err_msg=f"greedy, case {ci} rank {r}")


def test_sharded_matches_full_layer_on_two_gloo_ranks():
    _run_world(2, CASES)


@pytest.mark.parametrize("world", [4, 8])
def test_sharded_ragged_and_empty_shards_on_many_gloo_ranks(world):
    _run_world(world, CASES_WIDE)


def test_single_process_is_unsharded():
    p, s, z, idx, ow, bias = _layer(64, 64, 3, 9)
    lin = ShardedW4A16Linear(p, s, z, outlier_idx=idx, outlier_w=ow, bias=bias, marlin_layout=True,
                             device=torch.device("cpu"), local_fn=_oracle_local, argmax_fn=_oracle_argmax)
    assert lin.world == 1 and lin.rows == 64
    x = torch.randn(1, 64).to(torch.float16)
    full = _oracle_local(x, p, s, z, idx, ow, bias, True).numpy()
    np.testing.assert_array_equal(lin(x).numpy(), full)
    assert int(lin.greedy(x)) == int(np.argmax(full.astype(np.float32)))
