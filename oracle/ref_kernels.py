"""The reference's own device kernels, run on the GPU (TEST INFRASTRUCTURE).

Loads ``oracle/_ref/libqtts_ref.so`` (built by ``oracle/build_ref.py`` from the
kernel sources of the reference's ``src/gpu/kernels.rs``) and composes its
kernels the way the reference does, so tests can compare the oracle
restatement (``oracle/qtts_oracle.py``) with outputs of the reference itself.

* ``RefKernels`` -- one method per reference kernel launch (device tensors).
* ``RefDecodeStack`` -- ``decode_step_layer_on_stream``
  (``src/model/decode.rs:1694-1894``): the reference's kernel sequence for one
  decode position, with its fp32 KV caches ``[kv_heads, max_steps, head_dim]``.
  The projections are ``sgemm_row_major`` (rocBLAS, ``src/gpu/blas.rs:72-153``)
  in the reference; here torch's fp32 matmul with TF32 disabled stands in for
  that library GEMM (same math, different summation order).
* ``ref_head_token`` -- ``compute_logits_and_token`` (``src/model/talker.rs:431-496``):
  final RMSNorm, head GEMM, repetition penalty, suppression, argmax or device
  top-k sampling.

Never imported by the product path.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

import numpy as np
import torch

LIB = Path(__file__).resolve().parent / "_ref" / "libqtts_ref.so"


def available() -> bool:
    return LIB.exists()


def _p(t: torch.Tensor):
    assert t.is_cuda and t.is_contiguous()
    return C.c_void_p(t.data_ptr())


class RefKernels:
    def __init__(self):
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} missing: run python oracle/build_ref.py")
        self.lib = C.CDLL(str(LIB))

    def _ok(self, rc: int):
        if rc != 0:
            raise RuntimeError(f"reference kernel launch failed with cudaError {rc}")

    def rmsnorm(self, x, gamma, eps, rows, cols):
        out = torch.empty_like(x)
        self._ok(self.lib.ref_rmsnorm(_p(x), _p(gamma), _p(out), rows, cols, C.c_float(eps)))
        return out

    def rope(self, x, heads, steps, head_dim, offset, theta):
        out = torch.empty_like(x)
        self._ok(self.lib.ref_rope(_p(x), _p(out), x.numel(), heads, steps, head_dim, offset,
                                   C.c_float(theta)))
        return out

    def write_kv(self, x, cache, heads, input_steps, cache_steps, head_dim, offset):
        self._ok(self.lib.ref_write_kv(_p(x), _p(cache), heads, input_steps, cache_steps,
                                       head_dim, offset))

    def scores_cache(self, q, k, q_heads, kv_heads, key_steps, cache_steps, head_dim, offset,
                     scale):
        out = torch.empty(q_heads * key_steps, device=q.device, dtype=torch.float32)
        self._ok(self.lib.ref_attention_scores_cache(_p(q), _p(k), _p(out), q_heads, kv_heads, 1,
                                                     key_steps, cache_steps, head_dim, offset,
                                                     C.c_float(scale)))
        return out

    def softmax(self, x, rows, cols):
        out = torch.empty_like(x)
        self._ok(self.lib.ref_softmax(_p(x), _p(out), rows, cols))
        return out

    def apply_value_cache(self, probs, v, q_heads, kv_heads, key_steps, cache_steps, head_dim):
        out = torch.empty(q_heads * head_dim, device=probs.device, dtype=torch.float32)
        self._ok(self.lib.ref_apply_value_cache(_p(probs), _p(v), _p(out), q_heads, kv_heads, 1,
                                                key_steps, cache_steps, head_dim))
        return out

    def residual_add(self, a, b):
        out = torch.empty_like(a)
        self._ok(self.lib.ref_residual_add(_p(a), _p(b), _p(out), a.numel()))
        return out

    def swiglu(self, gate, up):
        out = torch.empty_like(gate)
        self._ok(self.lib.ref_swiglu(_p(gate), _p(up), _p(out), gate.numel()))
        return out

    def argmax(self, logits) -> int:
        out = torch.zeros(1, device=logits.device, dtype=torch.int32)
        self._ok(self.lib.ref_argmax(_p(logits), _p(out), logits.numel()))
        return int(out.item())

    def suppress(self, logits, eos):
        out = torch.empty_like(logits)
        self._ok(self.lib.ref_suppress(_p(logits), _p(out), logits.numel(), eos))
        return out

    def penalty(self, logits, tokens, penalty):
        """In place, as the reference's kernel."""
        t = torch.as_tensor(np.asarray(tokens, dtype=np.int32), device=logits.device)
        self._ok(self.lib.ref_penalty(_p(logits), _p(t), t.numel(), logits.numel(),
                                      C.c_float(penalty)))
        return logits

    def sample_topk(self, logits, top_k, temperature, u) -> int:
        out = torch.zeros(1, device=logits.device, dtype=torch.int32)
        self._ok(self.lib.ref_sample_topk(_p(logits), _p(out), logits.numel(), top_k,
                                          C.c_float(temperature), C.c_float(u)))
        return int(out.item())


def sgemm_row(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y[1, N] = x[1, K] . W[N, K]^T in fp32 (the rocBLAS sgemm_row_major stand-in)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (x.view(1, -1) @ w.T).view(-1).contiguous()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


class RefDecodeStack:
    """The reference's decode step over N layers, kernel by kernel
    (decode_step_layer_on_stream, src/model/decode.rs:1694-1894)."""

    def __init__(self, oracle_stack, device="cuda"):
        self.k = RefKernels()
        self.d = oracle_stack.d
        self.max_steps = oracle_stack.max_steps
        self.layers = []
        for L in oracle_stack.layers:
            dl = {n: t.to(device).contiguous() for n, t in L.items()}
            dl["qkv"] = torch.cat([dl["q"], dl["k"], dl["v"]]).contiguous()
            dl["gate_up"] = torch.cat([dl["gate"], dl["up"]]).contiguous()
            self.layers.append(dl)
        d = self.d
        self.k_cache = [torch.zeros(d.kv_heads * self.max_steps * d.head_dim, device=device)
                        for _ in self.layers]
        self.v_cache = [torch.zeros_like(c) for c in self.k_cache]

    def layer(self, li: int, x: torch.Tensor, offset: int) -> torch.Tensor:
        d, L, k = self.d, self.layers[li], self.k
        q_out, kv_out = d.q_heads * d.head_dim, d.kv_heads * d.head_dim
        active = offset + 1
        scale = np.float32(1.0 / math.sqrt(d.head_dim))
        normed = k.rmsnorm(x, L["in_g"], d.eps, 1, d.hidden)
        qkv = sgemm_row(normed, L["qkv"])
        q, kk, v = qkv[:q_out].contiguous(), qkv[q_out:q_out + kv_out].contiguous(), \
            qkv[q_out + kv_out:].contiguous()
        qn = k.rmsnorm(q, L["q_g"], d.eps, d.q_heads, d.head_dim)
        kn = k.rmsnorm(kk, L["k_g"], d.eps, d.kv_heads, d.head_dim)
        qr = k.rope(qn, d.q_heads, 1, d.head_dim, offset, d.theta)
        kr = k.rope(kn, d.kv_heads, 1, d.head_dim, offset, d.theta)
        k.write_kv(kr, self.k_cache[li], d.kv_heads, 1, self.max_steps, d.head_dim, offset)
        k.write_kv(v, self.v_cache[li], d.kv_heads, 1, self.max_steps, d.head_dim, offset)
        scores = k.scores_cache(qr, self.k_cache[li], d.q_heads, d.kv_heads, active,
                                self.max_steps, d.head_dim, offset, float(scale))
        probs = k.softmax(scores, d.q_heads, active)
        att = k.apply_value_cache(probs, self.v_cache[li], d.q_heads, d.kv_heads, active,
                                  self.max_steps, d.head_dim)
        h1 = k.residual_add(x, sgemm_row(att, L["o"]))
        post = k.rmsnorm(h1, L["post_g"], d.eps, 1, d.hidden)
        gu = sgemm_row(post, L["gate_up"])
        act = k.swiglu(gu[:d.intermediate].contiguous(), gu[d.intermediate:].contiguous())
        return k.residual_add(h1, sgemm_row(act, L["down"]))

    def step(self, x: torch.Tensor, offset: int) -> torch.Tensor:
        for li in range(len(self.layers)):
            x = self.layer(li, x, offset)
        return x


def ref_head_token(k: RefKernels, pre_norm, norm_g, head_w, eps, history, penalty, eos,
                   sample=None):
    """compute_logits_and_token_with_options (src/model/talker.rs:431-496):
    final norm -> head GEMM -> per-occurrence penalty -> suppression -> token.
    ``sample`` = (top_k, temperature, u) for device top-k, else argmax.
    Returns (raw logits, processed logits, token) as host arrays."""
    hidden = k.rmsnorm(pre_norm, norm_g, eps, 1, pre_norm.numel())
    logits = sgemm_row(hidden, head_w)
    raw = logits.clone()
    if history is not None and len(history) and penalty != 1.0:
        k.penalty(logits, history, penalty)
    sup = k.suppress(logits, eos)
    tok = k.argmax(sup) if sample is None else k.sample_topk(sup, *sample)
    return raw.cpu().numpy(), sup.cpu().numpy(), tok
