"""Row-sharded linear on GPUs: 2 NCCL ranks (one per GPU), each computing its
rows with the CUDA kernels, must assemble the full layer's output -- the same
on every rank and within the GEMV / GEMM parity bars of the oracle's result
(M = 1 and M = 32, ragged last shard, outliers, bias); the sharded greedy
head picks the first maximum of that output.  Needs >= 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CASES = [  # (N, K, n_out, M, seed)
    (4099, 2048, 21, 1, 1),
    (4099, 2048, 21, 32, 2),
    (8192, 4096, 41, 1, 3),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(N, K, n_out, seed):
    from tests.helpers import random_format
    f = random_format(N, K, n_out, seed=seed, ow_dtype="bf16")
    g = torch.Generator().manual_seed(seed)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    return f, bias


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from spectra_b200.sharded import ShardedW4A16Linear
        out = []
        for N, K, n_out, M, seed in CASES:
            f, bias = _layer(N, K, n_out, seed)
            lin = ShardedW4A16Linear(torch.from_numpy(f["packed"]), torch.from_numpy(f["scales"]),
                                     torch.from_numpy(f["zeros"]), outlier_idx=torch.from_numpy(f["outlier_idx"]),
                                     outlier_w=f["outlier_w_t"], bias=bias, marlin_layout=True,
                                     device=torch.device("cuda", rank))
            x = torch.randn(M, K, generator=torch.Generator().manual_seed(seed + 7)).to(torch.bfloat16)
            y = lin.forward(x.cuda(rank))
            tok = lin.greedy(x.cuda(rank))
            torch.cuda.synchronize()
            out.append((y.float().cpu().numpy(), tok.cpu().numpy()))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_layer_on_two_gpus_matches_oracle():
    from oracle import w4a16 as O
    from tests.helpers import assert_close_to_oracle, np_of
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for i, (N, K, n_out, M, seed) in enumerate(CASES):
        (y0, t0), (y1, t1) = res[0][i], res[1][i]
        assert np.array_equal(y0, y1), f"ranks disagree on case {i}"
        # the (value, index) reduction picks the first maximum of the gathered row
        assert np.array_equal(t0, t1) and np.array_equal(t0, np.argmax(y0, axis=-1)), f"greedy, case {i}"
        f, bias = _layer(N, K, n_out, seed)
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(seed + 7)).to(torch.bfloat16)
        ow, owd = np_of(f["outlier_w_t"])
        bn, bd = np_of(bias)
        for m in range(M):
            xn, xd = np_of(x[m:m + 1])
            if M == 1:
                y_exact, y_round, od = O.gemv(xn, xd, f["packed"], f["scales"], f["zeros"], bias=bn, bias_dtype=bd,
                                              outlier_idx=f["outlier_idx"], outlier_w=ow, ow_dtype=owd, marlin=True)
                assert_close_to_oracle(y0[m].astype(np.float64), y_exact, y_round, od, f"case {i}")
            else:
                c_exact, c_round, od = O.gemm(xn, xd, f["packed"], f["scales"], f["zeros"],
                                              outlier_idx=f["outlier_idx"], outlier_w=ow, ow_dtype=owd, marlin=True)
                ref = np.asarray(c_exact, np.float64).reshape(-1) + bias.double().numpy()
                err = np.max(np.abs(y0[m].astype(np.float64) - ref))
                assert err <= 1e-2 * np.max(np.abs(ref)), f"case {i} row {m}: {err}"
