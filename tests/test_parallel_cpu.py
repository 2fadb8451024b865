"""Host logic of the N-split exchange (qwen3-vl-2b-inference_b200/parallel.py)
on CPU: world_size-2 gloo process groups, a float reference product in place
of the GPU kernel.  Checks that the gathered result equals the unsplit one
exactly and that the 8-byte greedy exchange reproduces the reference's
greedy_decode (first index of the maximum, NaN never wins)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import import_qvl


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import importlib.util
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "qwen3-vl-2b-inference_b200")
    spec = importlib.util.spec_from_file_location("qvl_par", os.path.join(pkg, "parallel.py"))
    par = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(par)
    g = torch.Generator().manual_seed(0)
    if case == "gather":
        M, N, K = 5, 37, 16
        x = torch.randn(M, K, generator=g)
        W = torch.randint(-127, 128, (N, K), generator=g).float()
        S = torch.rand(N, generator=g)
        a, b = par.shard_rows(N, world, rank)
        fn = lambda xx, ww, ss: xx @ (ww * ss[:, None]).T   # noqa: E731
        C = par.split_linear_gather(x, W[a:b], S[a:b], N, fn)
        out_q.put((rank, bool(torch.equal(C, fn(x, W, S)))))
    else:
        R, N = 6, 23
        logits = torch.randn(R, N, generator=g)
        logits[0, [3, 17]] = 9.0            # tie across shards -> first index
        logits[1, :] = float("nan")
        logits[1, 20] = 1.0                  # NaN never wins
        logits[2, :] = float("-inf")         # no candidate -> 0
        logits[3, 11] = logits[3, 12] = 50.0 # tie inside one shard
        a, b = par.shard_rows(N, world, rank)
        got = par.split_greedy(logits[:, a:b], a)
        want = []
        for r in range(R):
            mv, mi = -np.finfo(np.float32).max, 0
            for j, v in enumerate(logits[r].tolist()):
                if v > mv:
                    mv, mi = v, j
            want.append(mi)
        out_q.put((rank, got.tolist() == want))
    dist.destroy_process_group()


@pytest.mark.parametrize("case", ["gather", "greedy"])
def test_nsplit_exchange_gloo_world2(case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res


def test_shard_rows_cover_exactly():
    import importlib.util
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "qwen3-vl-2b-inference_b200")
    spec = importlib.util.spec_from_file_location("qvl_par2", os.path.join(pkg, "parallel.py"))
    par = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(par)
    for n in (1, 7, 151936):
        for w in (1, 2, 3, 8):
            spans = [par.shard_rows(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(w - 1))
