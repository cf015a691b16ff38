"""Tensor-parallel decode-step projections across the GPUs of one node (one process per GPU).

Each projection is sharded on the dimension that keeps the layer's communication to ONE all-reduce of the
hidden vector per layer:

  * column-parallel (output rows split): QKV and gate_up. QKV is split by head groups (q, k and v rows of the
    same heads stay together) and gate_up by channel (gate row i and up row i land on the same rank), so the
    attention and silu(gate) * up that follow them need no exchange.
  * row-parallel (input columns split on 128-column group boundaries): o_proj and down. Each rank computes a
    partial output over its slice of K; the two partials are added and one all-reduce (sum) of the fp16
    hidden vector [H] completes the layer.

Shards keep the reference's weight format (kernels/int4_gemv.py:1-3): q uint8 [n, k/2], s and m fp16
[n, k/128]. A column split keeps whole rows; a row split keeps whole 128-column groups, so every shard is an
ordinary int4 GEMV operand for gemv_int4_cuda or Int4GemvSet.
"""
import torch

G = 128


def _span(n, rank, world, unit=1):
    """[lo, hi) of rank's share of n items, in whole units of `unit` items, as even as possible."""
    if n % unit:
        raise ValueError(f"{n} items do not split into units of {unit}")
    u = n // unit
    if u < world:
        raise ValueError(f"{n} items ({u} units of {unit}) cannot be split over {world} ranks")
    return (u * rank // world) * unit, (u * (rank + 1) // world) * unit


def shard_rows(w, rank, world, unit=1):
    """Column-parallel shard of an int4 matrix (q, s, m): a contiguous block of output rows."""
    q, s, m = w
    lo, hi = _span(q.shape[0], rank, world, unit)
    return q[lo:hi].contiguous(), s[lo:hi].contiguous(), m[lo:hi].contiguous()


def shard_cols(w, rank, world):
    """Row-parallel shard of an int4 matrix (q, s, m): a contiguous block of whole 128-column groups."""
    q, s, m = w
    g0, g1 = _span(s.shape[1], rank, world)
    return q[:, g0 * G // 2:g1 * G // 2].contiguous(), s[:, g0:g1].contiguous(), m[:, g0:g1].contiguous()


def col_span(K, rank, world):
    """[k0, k1) of the input columns that rank's row-parallel shard covers (whole 128-column groups)."""
    g0, g1 = _span(K // G, rank, world)
    return g0 * G, g1 * G


def _cat(parts):
    return tuple(torch.cat([p[i] for p in parts]).contiguous() for i in range(3))


def shard_qkv(w, rank, world, q_rows, kv_rows, head_dim=128):
    """Column-parallel QKV shard by head groups: rank r gets heads [lo, hi) of q and of k and of v."""
    q, s, m = w
    assert q.shape[0] == q_rows + 2 * kv_rows
    parts = []
    for base, rows in ((0, q_rows), (q_rows, kv_rows), (q_rows + kv_rows, kv_rows)):
        lo, hi = _span(rows, rank, world, head_dim)
        parts.append((q[base + lo:base + hi], s[base + lo:base + hi], m[base + lo:base + hi]))
    return _cat(parts)


def shard_gate_up(w, rank, world):
    """Column-parallel gate_up shard by channel: rank r gets gate rows [lo, hi) and the matching up rows."""
    q, s, m = w
    half = q.shape[0] // 2
    lo, hi = _span(half, rank, world)
    return _cat([(q[lo:hi], s[lo:hi], m[lo:hi]), (q[half + lo:half + hi], s[half + lo:half + hi],
                                                  m[half + lo:half + hi])])


def unshard_qkv(parts, world, q_rows, kv_rows, head_dim=128):
    """Full QKV output from the ranks' column shards (inverse of the shard_qkv row order)."""
    qs, ks, vs = [], [], []
    for r, y in enumerate(parts):
        nq = _span(q_rows, r, world, head_dim)
        nk = _span(kv_rows, r, world, head_dim)
        a, b = nq[1] - nq[0], nk[1] - nk[0]
        qs.append(y[:a]), ks.append(y[a:a + b]), vs.append(y[a + b:a + 2 * b])
    return torch.cat(qs + ks + vs)


def unshard_gate_up(parts, world):
    """Full gate_up output from the ranks' channel shards (inverse of the shard_gate_up row order)."""
    gates = [y[:y.shape[0] // 2] for y in parts]
    ups = [y[y.shape[0] // 2:] for y in parts]
    return torch.cat(gates + ups)


class TPLayerShards:
    """One decoder layer's projection shards on one rank (config-1 shapes: QKV = q 3072 + k 1024 + v 1024 rows,
    gate_up = 2 x 8192 rows, o_proj 3072 x 3072, down 3072 x 8192)."""

    def __init__(self, qkv, o, gate_up, down, rank, world, q_rows=3072, kv_rows=1024, head_dim=128):
        self.rank, self.world = rank, world
        self.qkv = shard_qkv(qkv, rank, world, q_rows, kv_rows, head_dim)
        self.gate_up = shard_gate_up(gate_up, rank, world)
        self.o = shard_cols(o, rank, world)
        self.down = shard_cols(down, rank, world)
        self.o_span = col_span(o[0].shape[1] * 2, rank, world)
        self.down_span = col_span(down[0].shape[1] * 2, rank, world)

    def partials(self, x_h, x_attn, x_act, gemv):
        """This rank's outputs: (qkv shard, gate_up shard, partial hidden = o partial + down partial).
        `gemv(x, q, s, m)` is any int4 GEMV with the reference's semantics."""
        y_qkv = gemv(x_h, *self.qkv)
        y_gu = gemv(x_h, *self.gate_up)
        k0, k1 = self.o_span
        d0, d1 = self.down_span
        part = gemv(x_attn[k0:k1].contiguous(), *self.o).float() + gemv(x_act[d0:d1].contiguous(), *self.down).float()
        return y_qkv, y_gu, part


class PeerAllReduce:
    """out = sum over the ranks of `group` of (a + b), for fp16 vectors of n elements: ONE kernel per call
    (rb_tp_allreduce_f16) that stores each rank's partial into every rank's buffer over NVLink and sums the
    slots in rank order, replacing the add kernel and the collective call of a row-parallel layer pair.
    Each rank's buffer comes from cudaMalloc (rb_ipc_alloc) and is mapped into the other ranks with CUDA IPC,
    opened for the mapping rank's own device with peer access enabled (rb_ipc_open): plain peer loads and
    stores, no multicast object. Every rank must make the same sequence
    of calls. Graph-capturable."""

    def __init__(self, n, device, group=None):
        import ctypes
        import torch.distributed as dist
        pg = group if group is not None else dist.group.WORLD
        self.world, self.rank, self.n = dist.get_world_size(pg), dist.get_rank(pg), n
        self.flag_off = (8 * self.world * n + 15) // 16 * 16
        self.counter_off = self.flag_off + 4 * 8
        from . import _lib
        L = _lib.lib()
        local, hbuf = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        with torch.cuda.device(device):
            _lib.check("rb_ipc_alloc", L.rb_ipc_alloc(self.counter_off + 16, ctypes.byref(local), hbuf))
        self._local = local.value
        metas = [None] * self.world
        dist.all_gather_object(metas, (hbuf.raw, 0), group=pg)
        self._bases = []  # mapped peer allocations, closed in close()
        ptrs = []
        with torch.cuda.device(device):
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._local)
                    continue
                handle, offset = metas[r]
                base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
                _lib.check("rb_ipc_open", L.rb_ipc_open(handle, offset, ctypes.byref(base), ctypes.byref(ptr)))
                self._bases.append(base.value)
                ptrs.append(ptr.value)
        self._bufs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=pg)

    def close(self):
        """Unmap the peers' buffers and free the local one (after every call that uses them has completed on
        every rank)."""
        from . import _lib
        for b in self._bases:
            _lib.lib().rb_ipc_close(b)
        self._bases = []
        if self._local:
            _lib.lib().rb_ipc_free(self._local)
            self._local = None

    def __call__(self, a, b, out):
        from . import _lib, config
        assert a.dtype == torch.float16 and out.dtype == torch.float16 and a.numel() == self.n == out.numel()
        st = _lib.lib().rb_tp_allreduce_f16(a.data_ptr(), None if b is None else b.data_ptr(), out.data_ptr(),
                                            self.n, self._bufs, self.rank, self.world, self.flag_off,
                                            self.counter_off, config.flags(), _lib.stream_ptr(a.device))
        _lib.check("rb_tp_allreduce_f16", st)
        return out


def allreduce_hidden(part, group=None):
    """Sum the ranks' partial hidden vectors (in place) with torch.distributed."""
    import torch.distributed as dist
    dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part


class TPDecodeStep:
    """A tensor-parallel decode step's projections on one rank, CUDA-graph capturable.

    Per layer: ONE multi-GEMV launch of the rank's four shards (QKV and gate_up on the layer input, o_proj and
    down on their slices of the attention and MLP activations), then the sum over ranks of o + down, which is
    the next layer's input: with collective="peer" one peer-memory reduction kernel (PeerAllReduce), with
    "nccl" an add kernel and an NCCL all-reduce. Then the int8 head, split by rows, and
    an all-gather of the logits. The attention and MLP activations are fixed inputs: the step covers the
    weight-only linear layers, which are the part this library implements.
    """

    def __init__(self, layers, x_attn, x_act, head, rank, world, group=None, q_rows=3072, kv_rows=1024,
                 collective="nccl"):
        from .gemv_set import Int4GemvSet
        dev = x_attn.device
        self.rank, self.world, self.group = rank, world, group
        self.ar = PeerAllReduce(x_attn.numel(), dev, group) if collective == "peer" and world > 1 else None
        H = x_attn.numel()
        self.h = [torch.zeros(H, device=dev, dtype=torch.float16) for _ in range(len(layers) + 1)]
        self.sets, self.outs = [], []
        for li, (qkv, o, gate_up, down) in enumerate(layers):
            sh = TPLayerShards(qkv, o, gate_up, down, rank, world, q_rows, kv_rows)
            k0, k1 = sh.o_span
            d0, d1 = sh.down_span
            xa = x_attn[k0:k1].contiguous()
            xi = x_act[d0:d1].contiguous()
            y_qkv = torch.empty(sh.qkv[0].shape[0], device=dev, dtype=torch.float16)
            y_gu = torch.empty(sh.gate_up[0].shape[0], device=dev, dtype=torch.float16)
            y_o = torch.empty(H, device=dev, dtype=torch.float16)
            y_d = torch.empty(H, device=dev, dtype=torch.float16)
            self.sets.append(Int4GemvSet([(self.h[li], *sh.qkv, y_qkv), (self.h[li], *sh.gate_up, y_gu),
                                          (xa, *sh.o, y_o), (xi, *sh.down, y_d)]))
            self.outs.append((y_qkv, y_gu, y_o, y_d, xa, xi, sh))
        hq, hs = head
        n = hq.shape[0]
        self.head_n = n
        self.head_rows = -(-n // world)
        lo, hi = min(n, rank * self.head_rows), min(n, (rank + 1) * self.head_rows)
        self.head = (hq[lo:hi].contiguous(), hs[lo:hi].contiguous())
        self.logits_part = torch.zeros(self.head_rows, device=dev, dtype=torch.float16)
        self.logits_all = torch.zeros(self.head_rows * world, device=dev, dtype=torch.float16)
        self.bytes = sum(s.bytes for s in self.sets) + hq[lo:hi].numel() + 2 * (hi - lo) + 2 * H + 2 * (hi - lo)

    def close(self):
        """Release the peer-memory reduction buffers (every rank, after its last step has completed)."""
        if self.ar is not None:
            self.ar.close()

    def __call__(self):
        import torch.distributed as dist
        from .cuda_gemv import gemv_int8_cuda
        for li, st in enumerate(self.sets):
            st()
            y_o, y_d = self.outs[li][2], self.outs[li][3]
            if self.ar is not None:
                self.ar(y_o, y_d, self.h[li + 1])
            else:
                torch.add(y_o, y_d, out=self.h[li + 1])
                if self.world > 1:
                    dist.all_reduce(self.h[li + 1], op=dist.ReduceOp.SUM, group=self.group)
        nrows = self.head[0].shape[0]
        if nrows:
            gemv_int8_cuda(self.h[-1], *self.head, out=self.logits_part[:nrows])
        if self.world > 1:
            dist.all_gather_into_tensor(self.logits_all, self.logits_part, group=self.group)
        else:
            self.logits_all.copy_(self.logits_part)
        return self.logits_all[:self.head_n]
