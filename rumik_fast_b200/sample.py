"""The sampling tail of a decode step in two launches (rb_sample): rumik-fast's FusedSampler (engine/sample.py).

    sampler = FusedSampler(eng, logits_fn)   # same constructor as engine/sample.py:91-113
    sampler()                                # logits_fn(), then writes eng.out[step], eng.tok, eng.step_i += 1

The maths is the reference's (engine/rumik_int4.py:174-198): the stop predictor
sigmoid(W2 . gelu(W1 . LayerNorm(hn) + b1) + b2) > 0.5 once min_new tokens are out, the </audio> row masked
before that, top_k (<= 32) of the head's logits and a Gumbel-max draw with uniforms from torch.rand (drawn
in-graph, as the reference does).
"""
import ctypes

import torch

from . import _lib, config
from .cuda_gemv import _on_device, _require


class FusedSampler:
    """eng: the engine (or any object) with hn, stop (dict of the stop predictor's tensors "0.weight", "0.bias",
    "1.weight", "1.bias", "3.weight", "3.bias"), audio_ids, end_id, step_i, tok, out, temperature, top_k,
    min_new, H and dev; logits_fn() returns the head's logits [>= len(audio_ids)]."""

    def __init__(self, eng, logits_fn):
        self.eng, self.logits_fn = eng, logits_fn
        d = eng.dev
        st = eng.stop
        self.lnw, self.lnb = st["0.weight"].float().contiguous(), st["0.bias"].float().contiguous()
        self.w1 = st["1.weight"].contiguous()
        self.b1 = st["1.bias"].float().contiguous()
        self.w2 = st["3.weight"].reshape(-1).float().contiguous()
        self.b2 = st["3.bias"].reshape(-1).float().contiguous()
        self.nz = self.w1.shape[0]
        self.nv = eng.audio_ids.numel()
        ends = (eng.audio_ids == eng.end_id).nonzero().flatten().tolist()
        _require(len(ends) == 1, "the head must hold </audio> exactly once")
        self.end_idx = ends[0]
        _require(1 <= eng.top_k <= 32, "top_k must be in 1..32")
        self.u = torch.empty(32, dtype=torch.float32, device=d)
        self.ws = torch.empty(_lib.lib().rb_sample_workspace(self.nz), dtype=torch.uint8, device=d)
        self.ids = eng.audio_ids.to(torch.int64).contiguous()

    def __call__(self):
        logits = self.logits_fn()
        torch.rand(32, device=self.eng.dev, out=self.u)  # graph-safe RNG (Philox offsets), as engine/sample.py:138
        return self.draw(logits)

    def draw(self, logits, u=None):
        """Sample from `logits` with the uniforms in self.u (or `u`, copied there first)."""
        e = self.eng
        if u is not None:
            self.u[:len(u)].copy_(u)
        for t in (logits, e.hn):
            _require(t.is_contiguous() and t.dtype in (torch.float16, torch.bfloat16, torch.float32),
                     "logits / hn must be contiguous fp16, bf16 or fp32")
        s = _lib.Sampler(logits.data_ptr(), _lib.dtype_code(logits.dtype), self.nv, self.end_idx,
                         self.ids.data_ptr(), e.top_k, 1.0 / e.temperature, self.u.data_ptr(), e.hn.data_ptr(),
                         _lib.dtype_code(e.hn.dtype), e.H, self.lnw.data_ptr(), self.lnb.data_ptr(),
                         self.w1.data_ptr(), _lib.dtype_code(self.w1.dtype), self.nz, self.b1.data_ptr(),
                         self.w2.data_ptr(), self.b2.data_ptr(), e.end_id, e.min_new, e.step_i.data_ptr(),
                         e.tok.data_ptr(), e.out.data_ptr(), e.out.numel(), self.ws.data_ptr())
        with _on_device(logits.device):
            st = _lib.lib().rb_sample(ctypes.byref(s), config.flags(), _lib.stream_ptr(logits.device))
        _lib.check("rb_sample", st)
        return e.tok[0]
