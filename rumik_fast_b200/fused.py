"""Decode-layer glue fused into the int4 GEMV launch (rb_gemv_int4_fused, rb_add_layernorm).

rumik-fast's decode step runs, per layer (engine/rumik_fused.py:84-116),

    gemv(h, w_in) -> post -> attention -> gemv(w_o), gemv(w_down) -> add_ln

where add_ln (engine/fused.py:29-40) forms the next residual x + o + down and its LayerNorm h, and post
(engine/fused.py:43-84) applies the rotary embedding, writes the new key/value to the cache and forms
silu(gate) * up. Here the add_ln runs inside the NEXT layer's input GEMV launch (every CTA normalises the
3072-element vector while it stages its activation tables) and post runs in that launch's epilogue (each
output row is routed to the query buffer, the caches or the MLP activation as it is produced), so the input
side of a layer is one kernel:

    layer = AddLnGemvPost(qkv, gate_up_interleaved, add_ln=AddLn(x, o_out, down_out, ln_w, x_next, eps), ...)
    layer()                       # add_ln + QKV GEMV + gate_up GEMV + rope + KV write + silu(gate) * up

Weights: the engine's fused w_in rows [q | k | v | gate | up] (engine/rumik_int4.py:95-100) are split with
split_w_in into the q|k|v rows (unchanged) and the gate|up rows re-ordered by interleave_gate_up (gate channel
c at row 2c, its up channel at row 2c + 1), so that the two rows of a channel finish in the same warp, like the
two elements of a rotary pair. Both are one-time permutations at load; the codes themselves are unchanged.

The residual stream alternates between two buffers (every CTA reads x while one CTA writes x + o + down).
"""
import ctypes

import torch

from . import _lib, config, scales8
from .cuda_gemv import _on_device, _require
from .gemv_set import _ws_len, _ws_ptr, workspace

G = 128


# ---------------------------------------------------------------------------------------------- weight layout
def gate_up_order(inter, device=None):
    """Row permutation of interleave_gate_up: new row r reads old row order[r] of [gate (inter) | up (inter)]."""
    c = torch.arange(inter, device=device)
    return torch.stack([c, c + inter], 1).reshape(-1)


def interleave_gate_up(q, s, m):
    """[gate; up] int4 rows (q [2I, K/2], s/m [2I, K/128]) -> the SwiGLU epilogue's order: gate channel c at row
    2c, its up channel at row 2c + 1."""
    _require(q.shape[0] % 2 == 0, f"gate_up rows {q.shape[0]} must be even")
    order = gate_up_order(q.shape[0] // 2, q.device)
    return q[order].contiguous(), s[order].contiguous(), m[order].contiguous()


def split_w_in(q, s, m, n_q_heads, n_kv_heads, head_dim):
    """The engine's fused w_in rows [q | k | v | gate | up] -> ((q, s, m) of q|k|v, (q, s, m) of gate|up in the
    SwiGLU order)."""
    nqkv = (n_q_heads + 2 * n_kv_heads) * head_dim
    _require(q.shape[0] > nqkv, "w_in has no MLP rows after q|k|v")
    qkv = tuple(t[:nqkv].contiguous() for t in (q, s, m))
    gu = interleave_gate_up(*(t[nqkv:] for t in (q, s, m)))
    return qkv, gu


# ---------------------------------------------------------------------------------------------- descriptors
class AddLn:
    """The add + LayerNorm prologue: x_out = x + a + b (fp32 sum, rounded once), h = LayerNorm(x_out) * w
    (engine/fused.py:29-40). a and b may be None; h_out (optional) receives h. AddLn.from_embedding builds the
    layer-0 form (engine/fused.py:18-27): the residual is the token's int8 embedding row times its scale."""

    def __init__(self, x, a, b, w, x_out, eps=1e-5, h_out=None):
        _require(x is not None, "x is required (AddLn.from_embedding builds the embedding form)")
        self._setup((x, a, b, w, x_out, h_out), eps)

    @classmethod
    def from_embedding(cls, emb_q, emb_s, tok, w, x_out, eps=1e-5, h_out=None):
        """emb_q int8 [vocab, H], emb_s [vocab] fp32/fp16, tok an int64 device tensor holding the token id."""
        _require(emb_q.dtype == torch.int8 and emb_q.dim() == 2 and emb_q.is_contiguous() and emb_q.is_cuda,
                 "emb_q must be a contiguous CUDA int8 [vocab, H] tensor")
        _require(emb_s.dtype in (torch.float32, torch.float16) and emb_s.numel() == emb_q.shape[0] and
                 emb_s.device == emb_q.device, "emb_s must hold one fp32/fp16 scale per embedding row")
        _require(tok.dtype == torch.int64 and tok.device == emb_q.device, "tok must be an int64 device tensor")
        _require(emb_q.shape[1] == w.numel(), "embedding rows must have H = w.numel() elements")
        self = cls.__new__(cls)
        self._setup((None, None, None, w, x_out, h_out), eps)
        self.c.emb_q, self.c.emb_s, self.c.tok = emb_q.data_ptr(), emb_s.data_ptr(), tok.data_ptr()
        self.c.vocab = emb_q.shape[0]
        self.c.emb_s_dtype = _lib.dtype_code(emb_s.dtype)
        self.embedding = (emb_q, emb_s, tok)
        return self

    def _setup(self, tensors, eps):
        x, a, b, w, x_out, h_out = tensors
        H, dt, dev = w.numel(), w.dtype, w.device
        for t, nm in zip(tensors, ("x", "a", "b", "w", "x_out", "h_out")):
            if t is None:
                continue
            _require(t.is_cuda and t.device == dev, f"{nm} must be on w's CUDA device")
            _require(t.dtype == dt and t.numel() == H and t.is_contiguous(),
                     f"{nm} must be a contiguous [{H}] {dt} vector")
        _require(H % G == 0 and H <= 12288, f"H={H} must be a multiple of {G} and <= 12288")
        self.tensors = tensors
        self.H, self.eps, self.dtype, self.device = H, float(eps), dt, dev
        ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        self.c = _lib.AddLn(ptr(x), ptr(a), ptr(b), ptr(w), ptr(x_out), ptr(h_out), H, self.eps)


def add_layernorm(ln: AddLn):
    """Run the add + LayerNorm on its own (the final norm in front of the head)."""
    with _on_device(ln.device):
        st = _lib.lib().rb_add_layernorm(ctypes.byref(ln.c), _lib.dtype_code(ln.dtype), config.flags(),
                                         _lib.stream_ptr(ln.device))
    _lib.check("rb_add_layernorm", st)


def _int4(w, K=None):
    """(q, s, m) with fp16 scale and min, or (q, scales8.Scales8, None) -> (descriptor of the GEMV with x and y
    unset, HBM bytes of its weights)."""
    q, s, m = w
    N, Kq = q.shape[0], q.shape[1] * 2
    _require(q.dtype == torch.uint8 and q.is_contiguous() and q.is_cuda, "q must be contiguous CUDA uint8 [N, K/2]")
    _require(K is None or Kq == K, f"weights have K={Kq}, activations {K}")
    if isinstance(s, scales8.Scales8):
        _require(m is None, "with 8-bit scales m must be None")
        scales8.check(s, N, Kq // G, q.device)
        d = _lib.GemvDesc(None, None, q.data_ptr(), s.sz.data_ptr(), None, N, Kq)
        d.s_row = s.s_row.data_ptr()
        return d, q.numel() + 2 * s.sz.numel() + 4 * s.s_row.numel()
    for t, nm in ((s, "s"), (m, "m")):
        _require(t.dtype == torch.float16 and t.is_contiguous() and tuple(t.shape) == (N, Kq // G),
                 f"{nm} must be a contiguous fp16 [{N}, {Kq // G}] tensor")
    return _lib.GemvDesc(None, None, q.data_ptr(), s.data_ptr(), m.data_ptr(), N, Kq), q.numel() + 4 * s.numel()


class AddLnGemvPost:
    """One decode layer's input side as ONE launch: [add_ln ->] gemv(w_qkv), gemv(w_gate_up) -> post.

    qkv      (q, s, m) of the q|k|v rows, N = (n_q_heads + 2 n_kv_heads) head_dim; or (q, Scales8, None) with
             8-bit scales (rumik_fast_b200.scales8: the launch then runs on the tcgen05 kernel)
    gate_up  (q, s, m) of the gate|up rows in interleave_gate_up order (or (q, Scales8, None), packed after
             interleaving)
    add_ln   an AddLn (its h is the GEMV input), or None with h = the input vector
    pos      int64 [1] device tensor: the position (cache slot) of this token
    cos, sin [cache_len, head_dim] rotary tables (engine/rumik_int4.py:107-109)
    k_cache, v_cache  [n_kv_heads, cache_len, head_dim];  q_out [n_q_heads * head_dim];  act [inter]
    rope     False for the layers without position embedding
    y_qkv, y_gate_up  optional buffers that also receive the plain GEMV results
    kernel   None (by size: the warp-MMA kernel for a layer's projections), "tc" or "mma"
    Built once (graph-capture safe to call); every tensor must stay alive.
    """

    def __init__(self, qkv, gate_up, *, pos, cos, sin, k_cache, v_cache, q_out, act, n_q_heads, n_kv_heads,
                 add_ln=None, h=None, rope=True, y_qkv=None, y_gate_up=None, kernel=None):
        _require((add_ln is None) != (h is None), "give exactly one of add_ln and h")
        src = add_ln.tensors[3] if add_ln is not None else h  # the norm weight: the activations' dtype
        self.device, self.x_dtype = src.device, src.dtype
        H = src.numel()
        dt = act.dtype
        _require(dt in (torch.float16, torch.bfloat16), "act must be fp16 or bf16")
        for t, nm in ((cos, "cos"), (sin, "sin"), (k_cache, "k_cache"), (v_cache, "v_cache"), (q_out, "q_out")):
            _require(t.dtype == dt and t.is_contiguous() and t.device == self.device,
                     f"{nm} must be a contiguous {dt} tensor on {self.device}")
        _require(pos.dtype == torch.int64 and pos.device == self.device, "pos must be an int64 tensor on the device")
        nkv, S, hd = k_cache.shape
        _require(nkv == n_kv_heads and tuple(v_cache.shape) == (nkv, S, hd), "caches must be [n_kv_heads, S, hd]")
        _require(tuple(cos.shape) == (S, hd) and tuple(sin.shape) == (S, hd), f"cos/sin must be [{S}, {hd}]")
        _require(q_out.numel() == n_q_heads * hd, "q_out must hold n_q_heads * head_dim elements")
        d_qkv, b_qkv = _int4(qkv, H)
        d_gu, b_gu = _int4(gate_up, H)
        Nqkv, Ngu = d_qkv.N, d_gu.N
        _require(Nqkv == (n_q_heads + 2 * n_kv_heads) * hd, "qkv rows must be (n_q_heads + 2 n_kv_heads) head_dim")
        _require(Ngu % 2 == 0 and act.numel() == Ngu // 2, "act must hold the N/2 MLP channels")
        for y, N in ((y_qkv, Nqkv), (y_gate_up, Ngu)):
            _require(y is None or (y.dtype == dt and y.numel() == N and y.is_contiguous()), "bad y buffer")
        xp = None if add_ln is not None else h.data_ptr()
        yp = lambda y: y.data_ptr() if y is not None else None  # noqa: E731
        descs = (_lib.GemvDesc * 2)(d_qkv, d_gu)
        for d, y in ((descs[0], y_qkv), (descs[1], y_gate_up)):
            d.x, d.y = xp, yp(y)
        epis = (_lib.GemvEpi * 2)()
        epis[0] = _lib.GemvEpi(_lib.EPI_ROPE_KV, int(bool(rope)), n_q_heads, n_kv_heads, hd, S, pos.data_ptr(),
                               cos.data_ptr(), sin.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(),
                               v_cache.data_ptr(), None)
        epis[1] = _lib.GemvEpi(_lib.EPI_SWIGLU, 0, 0, 0, 0, 0, None, None, None, None, None, None, act.data_ptr())
        self._descs, self._epis, self._ln = descs, epis, add_ln
        self.kflags = _lib.KERNEL_FLAGS[kernel]
        self.ws = workspace(descs, 2, self.device, self.kflags)
        self._keep = (qkv, gate_up, pos, cos, sin, k_cache, v_cache, q_out, act, h, y_qkv, y_gate_up)
        self.y_dtype = dt
        self.bytes = b_qkv + b_gu

    def __call__(self):
        L = _lib.lib()
        lnp = ctypes.byref(self._ln.c) if self._ln is not None else None
        with _on_device(self.device):
            st = L.rb_gemv_int4_fused(self._descs, self._epis, 2, lnp, None, _ws_ptr(self.ws), _ws_len(self.ws),
                                      _lib.dtype_code(self.x_dtype), _lib.dtype_code(self.y_dtype),
                                      config.flags() | self.kflags, _lib.stream_ptr(self.device))
        _lib.check("rb_gemv_int4_fused", st)


class AttnGemvSet:
    """A decode layer's output side as ONE launch: the decode attention over the KV cache (as
    attention.DecodeAttention) fused with the GEMVs that read its output (o_proj) and the ones that do not
    (down_proj, whose input is ready at launch and streams while the attention runs).

    entries  (x, q, s, m, y) as Int4GemvSet; entries whose x is `out` read the attention output, which the launch
             also stores to `out` (they are run after the others)
    q, k_cache, v_cache, pos, out, n_q_heads, n_kv_heads, scale: as DecodeAttention (1..4 query heads per
             key-value head)
    Runs on the warp-MMA GEMV kernel. Built once (graph-capture safe to call); every tensor must stay alive.
    """

    def __init__(self, entries, *, q, k_cache, v_cache, pos, out, n_q_heads, n_kv_heads, scale=None):
        from .gemv_set import Int4GemvSet
        reads = [e[0].data_ptr() == out.data_ptr() for e in entries]
        _require(any(reads), "no entry reads the attention output")
        ordered = [e for e, r in zip(entries, reads) if not r] + [e for e, r in zip(entries, reads) if r]
        self.set = Int4GemvSet(ordered, kernel="mma")  # validation and descriptors
        nkv, S, hd = k_cache.shape
        _require(nkv == n_kv_heads and tuple(v_cache.shape) == (nkv, S, hd), "caches must be [n_kv_heads, S, 128]")
        _require(n_q_heads % n_kv_heads == 0 and 1 <= n_q_heads // n_kv_heads <= 4,
                 "fused attention takes 1..4 query heads per key-value head")
        for t, nm in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (out, "out")):
            _require(t.is_cuda and t.dtype == self.set.x_dtype and t.is_contiguous(),
                     f"{nm} must be a contiguous {self.set.x_dtype} CUDA tensor")
        _require(q.numel() == n_q_heads * hd and out.numel() == n_q_heads * hd, "q/out must be [n_q_heads * hd]")
        _require(pos.dtype == torch.int64 and pos.device == q.device, "pos must be an int64 tensor on the device")
        need = _lib.lib().rb_attn_decode_workspace(n_q_heads, n_kv_heads, hd)
        _require(need > 0, f"unsupported heads {n_q_heads}/{n_kv_heads} x {hd}")
        self.ws = torch.zeros(need, dtype=torch.uint8, device=q.device)
        scale = float(hd ** -0.5 if scale is None else scale)
        self.src = _lib.AttnSrc(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                n_q_heads, n_kv_heads, hd, S, scale, self.ws.data_ptr(), need)
        self._keep = (q, k_cache, v_cache, pos, out)
        self.device = q.device
        self.bytes = self.set.bytes

    def __call__(self):
        s = self.set
        with _on_device(self.device):
            st = _lib.lib().rb_gemv_int4_fused(s._descs, None, len(s.entries), None, ctypes.byref(self.src), None, 0,
                                               _lib.dtype_code(s.x_dtype), _lib.dtype_code(s.y_dtype),
                                               config.flags() | _lib.FLAG_KERNEL_MMA, _lib.stream_ptr(self.device))
        _lib.check("rb_gemv_int4_fused", st)
