"""N-split linear + NCCL all-gather on 2 GPUs (skipped with fewer): every
output column computed on its owner rank must equal the single-GPU product
bit for bit, and the 8-byte-per-row greedy exchange must give the same token
as greedy_decode on the full logits."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import bench
    qvl = bench.import_qvl()
    import qvl_b200.parallel as par
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    g = torch.Generator().manual_seed(5)
    M, N, K = 4, 20000, 2048
    x = torch.randn(M, K, generator=g).to(dev)
    W = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g).to(dev)
    S = (torch.rand(N, generator=g) * 0.019 + 0.001).to(dev)
    a, b = par.shard_rows(N, world, rank)
    lin = lambda xx, ww, ss: qvl.linear(xx, ww.contiguous(), ss.contiguous(), group_quantized=False,  # noqa: E731
                                        semantics=qvl.SEM_LANE8)
    C = par.split_linear_gather(x, W[a:b], S[a:b], N, lin)
    full = lin(x, W, S)
    tok = par.split_greedy(C[:, a:b], a)
    ref_tok = qvl.greedy_decode(full).long()
    ok = bool(torch.equal(C, full)) and bool(torch.equal(tok.cpu(), ref_tok.cpu()))
    q.put((rank, ok))
    dist.destroy_process_group()


def _prefill_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import bench
    bench.import_qvl()
    import qvl_b200.decoder as D
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    cfg = D.TextConfig(layers=2)
    w = D.TextWeights.random(cfg, seed=7, device=dev)          # same values on every rank
    T = 452
    prompt = torch.randint(0, 151643, (T,), dtype=torch.int32, generator=torch.Generator().manual_seed(3)).to(dev)
    tp = D.TextDecoder(w, max_batch=1, max_ctx=T + 8, device=dev, tp_group=dist.group.WORLD)
    tp.prefill(prompt)
    one = D.TextDecoder(w, max_batch=1, max_ctx=T + 8, device=dev)
    one.prefill(prompt)
    torch.cuda.synchronize()
    ok = torch.equal(tp.logits, one.logits) and torch.equal(tp.tokens, one.tokens)
    ok = ok and all(torch.equal(a, b) for a, b in ((tp.k_all, one.k_all), (tp.v_all, one.v_all)))
    q.put((rank, bool(ok)))
    dist.destroy_process_group()


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return res


def test_prefill_tensor_split_two_gpus():
    """A 452-token prompt pass with every product split by output column over
    2 GPUs (NCCL all-gathers; the LM head's greedy token from the 8-byte
    exchange): logits, greedy token and the KV cache it leaves are identical
    to the single-GPU pass, bit for bit, on both ranks."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(_prefill_worker)
    assert all(ok for _, ok in res), res


def test_nsplit_linear_allgather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res
