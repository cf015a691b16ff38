"""Tensor-parallel sharding of the decode-step projections (rumik_fast_b200.tensor_parallel).

CPU tests: the shard arithmetic, and a world-size-2 gloo run in which every rank computes its shards' outputs
with the CPU oracle and the ranks all-reduce / gather them; the result must equal the unsharded oracle. The GPU
test runs every rank's shards through the CUDA kernels on one GPU and checks the recombined outputs."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O
from rumik_fast_b200 import tensor_parallel as tp

H, HEAD_DIM, Q_ROWS, KV_ROWS, INTER = 256, 64, 256, 128, 256   # small model: 4 q heads, 2 kv heads


def _weights(seed):
    rng = np.random.default_rng(seed)

    def w(n, k):
        q = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        s = rng.uniform(0.002, 0.02, size=(n, k // 128)).astype(np.float16)
        m = (-7.5 * s.astype(np.float32) + rng.normal(0, 1e-3, size=s.shape)).astype(np.float16)
        return torch.from_numpy(q), torch.from_numpy(s), torch.from_numpy(m)
    qkv, o, gu, down = w(Q_ROWS + 2 * KV_ROWS, H), w(H, H), w(2 * INTER, H), w(H, 2 * INTER)
    x_h = torch.from_numpy(rng.normal(0, 1, H).astype(np.float16))
    x_attn = torch.from_numpy(rng.normal(0, 1, H).astype(np.float16))
    x_act = torch.from_numpy(rng.normal(0, 1, 2 * INTER).astype(np.float16))
    return (qkv, o, gu, down), (x_h, x_attn, x_act)


def _oracle_gemv(x, q, s, m):
    return torch.from_numpy(O.gemv_int4_ref(x.numpy(), q.numpy(), s.numpy(), m.numpy()).astype(np.float32))


def _full_reference(W, X):
    (qkv, o, gu, down), (x_h, x_attn, x_act) = W, X
    return (_oracle_gemv(x_h, *qkv), _oracle_gemv(x_h, *gu),
            _oracle_gemv(x_attn, *o) + _oracle_gemv(x_act, *down))


def test_spans_cover_and_align():
    for n, unit in ((3072, 128), (1024, 128), (8192, 1), (24, 1)):
        for world in (1, 2, 4, 8):
            spans = [tp._span(n, r, world, unit) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(lo % unit == 0 and hi % unit == 0 for lo, hi in spans)
    with pytest.raises(ValueError):
        tp._span(1024, 0, 16, 128)          # 8 heads over 16 ranks
    with pytest.raises(ValueError):
        tp._span(100, 0, 2, 64)             # not whole units


def test_config_shapes_shard_on_group_boundaries():
    for world in (2, 4, 8):
        for K in (3072, 8192):
            spans = [tp.col_span(K, r, world) for r in range(world)]
            assert all(lo % 128 == 0 and hi % 128 == 0 for lo, hi in spans)
            assert sum(hi - lo for lo, hi in spans) == K


def test_shards_recombine_single_process():
    W, X = _weights(3)
    world = 2
    ref_qkv, ref_gu, ref_h = _full_reference(W, X)
    outs = []
    for r in range(world):
        sh = tp.TPLayerShards(*W, r, world, Q_ROWS, KV_ROWS, HEAD_DIM)
        outs.append(sh.partials(X[0], X[1], X[2], _oracle_gemv))
    qkv = tp.unshard_qkv([o[0] for o in outs], world, Q_ROWS, KV_ROWS, HEAD_DIM)
    gu = tp.unshard_gate_up([o[1] for o in outs], world)
    hidden = sum(o[2] for o in outs)
    assert torch.allclose(qkv, ref_qkv, rtol=1e-5, atol=1e-4)
    assert torch.allclose(gu, ref_gu, rtol=1e-5, atol=1e-4)
    assert torch.allclose(hidden, ref_h, rtol=1e-4, atol=1e-3)


def _gloo_rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, X = _weights(5)
        sh = tp.TPLayerShards(*W, rank, world, Q_ROWS, KV_ROWS, HEAD_DIM)
        y_qkv, y_gu, part = sh.partials(X[0], X[1], X[2], _oracle_gemv)
        tp.allreduce_hidden(part)
        qkv_parts = [torch.empty_like(y_qkv) for _ in range(world)]
        gu_parts = [torch.empty_like(y_gu) for _ in range(world)]
        dist.all_gather(qkv_parts, y_qkv)
        dist.all_gather(gu_parts, y_gu)
        if rank == 0:
            ref_qkv, ref_gu, ref_h = _full_reference(W, X)
            qkv = tp.unshard_qkv(qkv_parts, world, Q_ROWS, KV_ROWS, HEAD_DIM)
            gu = tp.unshard_gate_up(gu_parts, world)
            out["ok"] = bool(torch.allclose(qkv, ref_qkv, rtol=1e-5, atol=1e-4)
                             and torch.allclose(gu, ref_gu, rtol=1e-5, atol=1e-4)
                             and torch.allclose(part, ref_h, rtol=1e-4, atol=1e-3))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_gloo_world2():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = 29500 + (os.getpid() % 1000)
        procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert out.get("ok") is True


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_shards_through_cuda(native_lib, world):
    """Config-1 layer shapes: every rank's shards through the CUDA GEMV on one GPU, recombined."""
    from rumik_fast_b200 import gemv_int4_cuda, synthetic as syn
    from tests.helpers import assert_close
    dev = torch.device("cuda", 0)
    gen = syn.generator(11, dev)
    W = tuple(syn.int4_weights(n, k, gen, dev) for _, n, k in
              (("qkv", 5120, 3072), ("o", 3072, 3072), ("gate_up", 16384, 3072), ("down", 3072, 8192)))
    x_h, x_attn, x_act = (syn.activations((k,), gen, dev) for k in (3072, 3072, 8192))
    cpu = lambda t: t.cpu().numpy()
    ref_qkv = O.gemv_int4_ref(cpu(x_h), *map(cpu, W[0]))
    ref_gu = O.gemv_int4_ref(cpu(x_h), *map(cpu, W[2]))
    ref_h = O.gemv_int4_ref(cpu(x_attn), *map(cpu, W[1])) + O.gemv_int4_ref(cpu(x_act), *map(cpu, W[3]))
    gemv = lambda x, q, s, m: gemv_int4_cuda(x, q, s, m, out=torch.empty(q.shape[0], device=dev, dtype=torch.float16))
    outs = [tp.TPLayerShards(*W, r, world).partials(x_h, x_attn, x_act, gemv) for r in range(world)]
    qkv = tp.unshard_qkv([o[0] for o in outs], world, 3072, 1024)
    gu = tp.unshard_gate_up([o[1] for o in outs], world)
    hidden = sum(o[2] for o in outs)
    assert_close(qkv.float().cpu().numpy(), ref_qkv)
    assert_close(gu.float().cpu().numpy(), ref_gu)
    assert_close(hidden.cpu().numpy(), ref_h)


def _peer_rank(rank, world, port, out):
    import torch.distributed as dist
    from rumik_fast_b200 import device_error
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        n = 3072
        ar = tp.PeerAllReduce(n, dev)
        ok = True
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        outs, refs = [], []
        for it in range(5):  # several calls: both slot parities, epochs advancing
            a = (torch.randn(n, generator=g, device=dev) * (it + 1)).half()
            b = torch.randn(n, generator=g, device=dev).half()
            o = torch.empty(n, device=dev, dtype=torch.float16)
            ar(a, b, o)
            part = a.float() + b.float()
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            ref = parts[0].clone()
            for p_ in parts[1:]:
                ref += p_
            ok &= bool(torch.equal(o, ref.half()))
        # graph replay of three calls
        a = torch.randn(n, generator=g, device=dev).half()
        b = torch.randn(n, generator=g, device=dev).half()
        os_ = [torch.empty(n, device=dev, dtype=torch.float16) for _ in range(3)]
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for o in os_:
                ar(a, b, o)
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        part = a.float() + b.float()
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        ref = parts[0].clone()
        for p_ in parts[1:]:
            ref += p_
        ok &= all(bool(torch.equal(o, ref.half())) for o in os_)
        ok &= device_error(dev) == 0
        out[rank] = ok
        del gr
        torch.cuda.synchronize()
        dist.barrier()
        ar.close()
    finally:
        dist.destroy_process_group()


def _run_peer(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = 29700 + (os.getpid() % 200) + world
        procs = [ctx.Process(target=_peer_rank, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert all(out.get(r) is True for r in range(world)), dict(out)


@pytest.mark.gpu
def test_peer_allreduce_world1(native_lib):
    _run_peer(1)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_world2(native_lib):
    _run_peer(2)
