"""The exact kernel instance the headline benchmark times, at the size it is timed.

bench.py's decode workload runs the 36-layer config-1 projection set (144 GEMVs, 7,776 blocks of 128 rows) and
the int8 head's rows (16385 x 3072, 129 blocks, the list's last entry) as one Int4GemvSet launch. That list is far longer than
3 x the SM count, so it runs on the tcgen05 kernel UNSPLIT: each CTA walks about 53 blocks and every ring slot and
tensor-memory buffer wraps its phase many times.
These tests build that list (distinct weights per layer, as the bench does, but a distinct output per entry so
that every entry can be checked), run it twice, and compare every output row of every entry with the fp32
oracle (kernels/bench_cuda.py:38's check, dequantize(q, s, m) @ x.float(), in the multi-threaded torch
restatement oracle/reference_cpu.py). Whole outputs, not row samples: a bf16 output compared on a few hundred
rows is dominated by single rounding flips (tests/helpers.py:assert_close).
"""
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import reference_cpu as R
from rumik_fast_b200 import synthetic as syn
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rb.device_error()
    yield
    assert rb.device_error() == 0


def check_all(ent, what):
    for i, (x, q, s, m, y) in enumerate(ent):
        if m is None:  # the int8 head's rows
            ref = R.gemv_int8_torch(x.cpu(), q.cpu(), s.cpu(), signed=q.dtype == torch.int8).numpy()
            assert_close(y, ref, f"{what} entry {i}: int8 rows (N={q.shape[0]}, K={q.shape[1]})")
            continue
        ref = R.gemv_int4_torch(x.cpu(), q.cpu(), s.cpu(), m.cpu()).numpy()
        assert_close(y, ref, f"{what} entry {i} (N={q.shape[0]}, K={2 * q.shape[1]})")


def step_list(dtype, layers=36, seed=1234, head=True):
    """bench.py's step list: per layer QKV, o_proj, gate_up with x_h and down with x_i, then the int8 head's rows
    (int8 codes, fp16 row scales, x_h)."""
    gen = syn.generator(seed, DEV)
    xh = syn.activations((3072,), gen, DEV, dtype=dtype)
    xi = syn.activations((8192,), gen, DEV, dtype=dtype)
    ent = []
    head_entry = []
    if head:
        q8, s8 = syn.int8_weights(*syn.HEAD_SHAPE, gen, DEV)
        head_entry.append((xh, q8, s8, None, torch.full((syn.HEAD_SHAPE[0],), float("nan"), device=DEV,
                                                        dtype=dtype)))
    for _ in range(layers):
        for name, n, k in syn.LAYER_SHAPES:
            q, s, m = syn.int4_weights(n, k, gen, DEV)
            ent.append((xi if name == "down" else xh, q, s, m, torch.full((n,), float("nan"), device=DEV,
                                                                          dtype=dtype)))
    return ent + head_entry


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_whole_step_projection_set_unsplit(dtype):
    ent = step_list(dtype)
    st = rb.Int4GemvSet(ent)
    assert st.ws is None                                  # 129 + 7,776 blocks: never split
    assert sum((q.shape[0] + 127) // 128 for _, q, _, _, _ in ent) == 129 + 7776
    st()
    torch.cuda.synchronize()
    first = [e[4].clone() for e in ent]
    st()
    torch.cuda.synchronize()
    assert all(torch.equal(a, e[4]) for a, e in zip(first, ent)), "two calls differ"
    assert rb.device_error() == 0
    check_all(ent, "36-layer set")


def test_long_bands_tc_ring():
    """About 50 blocks per CTA at a short K (4 groups, 2 ring stages per block): every ring slot and
    tensor-memory buffer of each converter set wraps its phase dozens of times (the regression case of the
    phase-aliasing fault once met on long row bands, here on the tcgen05 kernel)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n_blocks = 50 * sms
    shapes = [(n_blocks // 4 * 128 - 77, 512)] * 3 + [(n_blocks // 4 * 128 + 5, 512)]
    gen = syn.generator(5, DEV)
    ent = []
    for n, k in shapes:
        q, s, m = syn.int4_weights(n, k, gen, DEV)
        ent.append((syn.activations((k,), gen, DEV), q, s, m, torch.full((n,), float("nan"), device=DEV,
                                                                        dtype=torch.float16)))
    st = rb.Int4GemvSet(ent, kernel="tc")
    assert st.ws is None
    st()
    st()
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    check_all(ent, "long bands")
