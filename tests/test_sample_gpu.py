"""The sampling tail (rb_sample / FusedSampler) on the GPU against the oracle and the reference's fixtures."""
import os
import types

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200.sample import FusedSampler
from tests.helpers import bf16_from_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden", "golden_glue.npz")


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rb.device_error()
    yield
    assert rb.device_error() == 0


def engine(hn, stop, ids, step, top_k=30, temperature=0.8, min_new=8, out_len=64):
    return types.SimpleNamespace(hn=hn, stop=stop, audio_ids=ids, end_id=int(ids[-1]), H=hn.numel(), dev=DEV,
                                 step_i=torch.tensor([step], device=DEV), tok=torch.zeros(1, dtype=torch.int64,
                                 device=DEV), out=torch.full((out_len,), -1, dtype=torch.int64, device=DEV),
                                 temperature=temperature, top_k=top_k, min_new=min_new)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_reference_cases(case):
    g = np.load(GOLD)
    step, min_new, top_k, end_idx, end_id = (int(v) for v in g[f"smp{case}_meta"])
    stop = {"0.weight": torch.from_numpy(g[f"smp{case}_lnw"]).to(DEV),
            "0.bias": torch.from_numpy(g[f"smp{case}_lnb"]).to(DEV),
            "1.weight": bf16_from_bits(g[f"smp{case}_w1"]).to(DEV),
            "1.bias": torch.from_numpy(g[f"smp{case}_b1"]).to(DEV),
            "3.weight": torch.from_numpy(g[f"smp{case}_w2"]).reshape(1, -1).to(DEV),
            "3.bias": torch.from_numpy(g[f"smp{case}_b2"]).to(DEV)}
    ids = torch.from_numpy(g["smp_ids"]).to(DEV)
    eng = engine(bf16_from_bits(g[f"smp{case}_hn"]).to(DEV), stop, ids, step, top_k=top_k, min_new=min_new)
    sampler = FusedSampler(eng, None)
    logits = bf16_from_bits(g[f"smp{case}_logits"]).to(DEV)
    sampler.draw(logits, torch.from_numpy(g[f"smp{case}_u"]).to(DEV))
    torch.cuda.synchronize()
    want = int(g[f"smp{case}_next"])
    assert eng.tok.item() == want and eng.out[step].item() == want and eng.step_i.item() == step + 1


@pytest.mark.parametrize("nv,top_k,dtype", [(16385, 30, torch.float32), (32768, 32, torch.float16),
                                            (1000, 1, torch.bfloat16), (31, 30, torch.float32)])
def test_random_cases_against_the_oracle(nv, top_k, dtype):
    gen = torch.Generator().manual_seed(nv + top_k)
    H, nz = 2048, 512
    ids = torch.randperm(100000, generator=gen)[:nv].to(torch.int64)
    for trial, (step, b2) in enumerate(((2, 4.0), (12, -4.0), (12, 4.0), (40, -4.0))):
        logits = (torch.randn(nv, generator=gen) * 3).to(dtype)
        hn = torch.randn(H, generator=gen).to(torch.bfloat16)
        stop = {"0.weight": 1 + 0.1 * torch.randn(H, generator=gen), "0.bias": 0.1 * torch.randn(H, generator=gen),
                "1.weight": (0.02 * torch.randn(nz, H, generator=gen)).to(torch.bfloat16),
                "1.bias": 0.1 * torch.randn(nz, generator=gen), "3.weight": 0.05 * torch.randn(1, nz, generator=gen),
                "3.bias": torch.tensor([b2])}
        u = torch.rand(32, generator=gen)
        eng = engine(hn.to(DEV), {k: v.to(DEV) for k, v in stop.items()}, ids.to(DEV), step, top_k=top_k)
        sampler = FusedSampler(eng, None)
        sampler.draw(logits.to(DEV), u.to(DEV))
        torch.cuda.synchronize()
        hn_np = hn.view(torch.int16).numpy().view(np.uint16)
        s = O.stop_logit_ref(hn_np, stop["0.weight"].numpy(), stop["0.bias"].numpy(),
                             stop["1.weight"].float().numpy(), stop["1.bias"].numpy(), stop["3.weight"].numpy(),
                             stop["3.bias"].numpy(), "bf16")
        want = O.pick_ref(logits.float().numpy(), step, 8, nv - 1, u.numpy(), top_k, np.float32(1 / 0.8),
                          ids.numpy(), s, int(ids[-1]))
        assert eng.tok.item() == want, f"trial {trial}"
        assert eng.step_i.item() == step + 1 and eng.out[step].item() == want


def test_in_a_cuda_graph_with_in_graph_uniforms():
    """Captured with torch.rand inside (as the engine does): each replay writes the next slot of out."""
    gen = torch.Generator().manual_seed(3)
    nv, H, nz = 16385, 2048, 512
    ids = torch.arange(nv, dtype=torch.int64, device=DEV) + 7
    stop = {"0.weight": torch.ones(H, device=DEV), "0.bias": torch.zeros(H, device=DEV),
            "1.weight": (0.02 * torch.randn(nz, H, generator=gen)).to(torch.bfloat16).to(DEV),
            "1.bias": torch.zeros(nz, device=DEV), "3.weight": torch.zeros(1, nz, device=DEV),
            "3.bias": torch.tensor([-1.0], device=DEV)}                    # never stops
    logits = torch.randn(nv, generator=gen).to(torch.float16).to(DEV)
    eng = engine(torch.randn(H, generator=gen).to(torch.bfloat16).to(DEV), stop, ids, 0)
    sampler = FusedSampler(eng, lambda: logits)
    sampler()
    torch.cuda.synchronize()
    eng.step_i.zero_()
    eng.out.fill_(-1)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sampler()
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    assert eng.step_i.item() == 5
    top = set((torch.topk(logits.float(), 30).indices + 7).tolist())
    got = eng.out[:5].tolist()
    assert all(t in top for t in got) and eng.out[5].item() == -1
