"""Row-sharded linear on GPUs: 2 NCCL ranks (one per GPU), each computing its
rows with the CUDA kernels, must assemble the full layer's output -- the same
on every rank and within the GEMV / GEMM parity bars of the oracle's result
(M = 1 and M = 32, ragged last shard, outliers, bias); the sharded greedy
head picks the first maximum of that output.  Both exchanges are run: the
peer-memory all-gather over NVLink (the default on NCCL groups) and the
group's own all-gather, and must agree bit for bit; the peer-memory path is
also captured in a CUDA graph and replayed on fresh inputs.  Needs >= 2 GPUs."""
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


def _x(M, K, seed):
    return torch.randn(M, K, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    layers = []
    try:
        from spectra_b200 import kernels as SK
        from spectra_b200.sharded import ShardedW4A16Linear
        SK.device_timeouts(reset=True)
        out = []
        for N, K, n_out, M, seed in CASES:
            f, bias = _layer(N, K, n_out, seed)
            res = {}
            for exchange in ("p2p", "collective"):
                lin = ShardedW4A16Linear(torch.from_numpy(f["packed"]), torch.from_numpy(f["scales"]),
                                         torch.from_numpy(f["zeros"]),
                                         outlier_idx=torch.from_numpy(f["outlier_idx"]), outlier_w=f["outlier_w_t"],
                                         bias=bias, marlin_layout=True, device=dev, exchange=exchange)
                layers.append(lin)
                assert lin.use_p2p == (exchange == "p2p")
                x = _x(M, K, seed + 7).to(dev)
                y = lin.forward(x)
                y2 = lin.forward(x)   # second call: the other buffer parity
                tok = lin.greedy(x)
                torch.cuda.synchronize()
                assert torch.equal(y, y2)
                res[exchange] = (y.float().cpu().numpy(), tok.cpu().numpy())
                if exchange == "p2p":
                    assert lin._exchanges[("y", M, torch.bfloat16)] is not None
                    # graph capture of the two-kernel call, replayed on new inputs
                    xs = x.clone()
                    lin.forward(xs), lin.greedy(xs)  # warm-up on the capture's shapes
                    torch.cuda.synchronize()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        yg = lin.forward(xs)
                        tg = lin.greedy(xs)
                    reps = []
                    for j in range(3):
                        xj = _x(M, K, 1000 * seed + j).to(dev)
                        xs.copy_(xj)
                        g.replay()
                        torch.cuda.synchronize()
                        reps.append((yg.clone(), tg.clone(), lin.forward(xj), lin.greedy(xj)))
                    for yr, tr, ye, te in reps:
                        assert torch.equal(yr, ye) and torch.equal(tr, te), "graph replay differs from eager"
                    del g
            out.append((res["p2p"], res["collective"]))
        torch.cuda.synchronize()
        out.append(SK.device_timeouts())
        q.put((rank, out))
    finally:
        for lin in layers:
            lin.close()
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
    assert res[0][-1] == 0 and res[1][-1] == 0, "a device wait timed out"
    for i, (N, K, n_out, M, seed) in enumerate(CASES):
        (y0, t0), (yc0, tc0) = res[0][i]
        (y1, t1), (yc1, tc1) = res[1][i]
        assert np.array_equal(y0, y1), f"ranks disagree on case {i}"
        # the peer-memory exchange and the group's all-gather assemble the same bits
        assert np.array_equal(y0, yc0) and np.array_equal(y1, yc1), f"exchanges differ, case {i}"
        assert np.array_equal(t0, tc0) and np.array_equal(t1, tc1)
        # the (value, index) reduction picks the first maximum of the gathered row
        assert np.array_equal(t0, t1) and np.array_equal(t0, np.argmax(y0, axis=-1)), f"greedy, case {i}"
        f, bias = _layer(N, K, n_out, seed)
        x = _x(M, K, seed + 7)
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
