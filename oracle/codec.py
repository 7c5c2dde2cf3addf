"""Codec decoder oracle: seeded synthetic weights + a PyTorch-CPU fp32 restatement.

TEST INFRASTRUCTURE. Nothing in the product path imports this file; tests,
``bench.py``'s reference arm and ``__graft_entry__.smoke()`` use it as the
checker for the CUDA codec decoder.

The reference decoder is ``HipCodecInitial`` (src/audio/codec_hip.rs): codes
[frames x 16] -> 24 kHz waveform, 1920 samples per frame. Its stages, restated
here in the same order and with the same formulas:

* RVQ (codec_rvq_project_f32, src/gpu/kernels.rs:454-497): normalised
  codebooks (embedding_sum / max(cluster_usage, 1e-7),
  codec_hip.rs:2135-2154); first codebook and the sum of the 15 rest
  codebooks, each through its 1x1 output projection, summed.
* pre_conv: causal conv 512 -> 1024, kernel 3, left pad 2
  (codec_causal_conv1d_f32, kernels.rs:499-529).
* pre_transformer (codec_hip.rs:379-653): input_proj 1024 -> 512 + bias,
  8 layers of RMSNorm (eps 1e-5) -> q/k/v (16 heads x 64) -> RoPE (theta 1e4,
  rotate-half, positions 0..T-1, kernels.rs:40-77) -> causal softmax attention
  (scale 1/8, kernels.rs:977-1014 and 120-174) -> o_proj, residual scaled by
  self_attn_layer_scale; RMSNorm -> SwiGLU MLP (1024) -> residual scaled by
  mlp_layer_scale; final RMSNorm; output_proj 512 -> 1024 + bias.
* two upsample stages (codec_hip.rs:656-785): transposed conv 1024 -> 1024,
  kernel 2, stride 2 (kernels.rs:662-692) then a ConvNeXt block: depthwise
  causal conv k 7 (pad 6), LayerNorm over channels (eps 1e-6), pwconv1
  1024 -> 4096, erf GELU, pwconv2 4096 -> 1024, residual + gamma * update.
* decoder (codec_hip.rs:787-1041): causal conv 1024 -> 1536 (k 7); 4 blocks
  (channels 1536->768->384->192->96, strides 8, 5, 4, 3): snake, transposed
  conv with kernel 2*stride keeping the first in*stride samples, three
  residual units (snake, dilated causal conv k 7 with dilation 1 / 3 / 9,
  snake, 1x1 conv, + input); final snake, causal conv 96 -> 1 (k 7), clamp to
  [-1, 1]. Snake: x + sin(x * e^alpha)^2 / (e^beta + 1e-9) (kernels.rs:731-749).

Synthetic weights (the real speech-tokenizer checkpoint is not available):
drawn from ``numpy.random.default_rng(seed)`` in sorted tensor-name order,
float32, scaled by 1/sqrt(fan-in) so activations stay O(1) through the stack
(conv2 of each residual unit at half that and the final conv at 1/20, so
the waveform's std is ~0.25 and few samples reach the clamp; layer scales
0.1, snake log-parameters N(0, 0.1), cluster usage U[0.5, 2], biases
N(0, 0.02), norm gammas 1 and betas 0). Parity is therefore unpinned to the
real model: it is pinned to this restatement of the reference's arithmetic.
"""
from __future__ import annotations

import json
import math
import struct
from pathlib import Path

import numpy as np

GROUPS = 16
CODEBOOK_SIZE = 2048
CODEBOOK_DIM = 256
PROJECTED = 512
PRE_CONV_OUT = 1024
HIDDEN = 512
LAYERS = 8
HEADS = 16
HEAD_DIM = 64
INTER = 1024
UP_CH = 1024
CONVNEXT_INTER = 4096
DECODER_INIT = 1536
BLOCKS = ((1536, 768, 8), (768, 384, 5), (384, 192, 4), (192, 96, 3))
DILATIONS = (1, 3, 9)
SAMPLES_PER_FRAME = 2 * 2 * 8 * 5 * 4 * 3  # 1920 at 24 kHz
SAMPLE_RATE = 24000


def tensor_specs() -> dict[str, tuple[tuple[int, ...], str, float]]:
    """name -> (shape, kind, scale); kind in normal/usage/one/zero/log/scale."""
    s: dict[str, tuple[tuple[int, ...], str, float]] = {}
    q = "decoder.quantizer"
    for name, n in (("rvq_first", 1), ("rvq_rest", GROUPS - 1)):
        for i in range(n):
            p = f"{q}.{name}.vq.layers.{i}._codebook"
            s[f"{p}.embedding_sum"] = ((CODEBOOK_SIZE, CODEBOOK_DIM), "normal", 1.0)
            s[f"{p}.cluster_usage"] = ((CODEBOOK_SIZE,), "usage", 0.0)
    s[f"{q}.rvq_first.output_proj.weight"] = ((PROJECTED, CODEBOOK_DIM, 1), "normal",
                                              1 / math.sqrt(CODEBOOK_DIM))
    s[f"{q}.rvq_rest.output_proj.weight"] = ((PROJECTED, CODEBOOK_DIM, 1), "normal",
                                             1 / math.sqrt(CODEBOOK_DIM * (GROUPS - 1)))
    s["decoder.pre_conv.conv.weight"] = ((PRE_CONV_OUT, PROJECTED, 3), "normal",
                                         1 / math.sqrt(PROJECTED * 3))
    s["decoder.pre_conv.conv.bias"] = ((PRE_CONV_OUT,), "normal", 0.02)
    t = "decoder.pre_transformer"
    s[f"{t}.input_proj.weight"] = ((HIDDEN, PRE_CONV_OUT), "normal", 1 / math.sqrt(PRE_CONV_OUT))
    s[f"{t}.input_proj.bias"] = ((HIDDEN,), "normal", 0.02)
    s[f"{t}.output_proj.weight"] = ((PRE_CONV_OUT, HIDDEN), "normal", 1 / math.sqrt(HIDDEN))
    s[f"{t}.output_proj.bias"] = ((PRE_CONV_OUT,), "normal", 0.02)
    s[f"{t}.norm.weight"] = ((HIDDEN,), "one", 0.0)
    qo = HEADS * HEAD_DIM
    for i in range(LAYERS):
        p = f"{t}.layers.{i}"
        s[f"{p}.input_layernorm.weight"] = ((HIDDEN,), "one", 0.0)
        for proj in ("q_proj", "k_proj", "v_proj"):
            s[f"{p}.self_attn.{proj}.weight"] = ((qo, HIDDEN), "normal", 1 / math.sqrt(HIDDEN))
        s[f"{p}.self_attn.o_proj.weight"] = ((HIDDEN, qo), "normal", 1 / math.sqrt(qo))
        s[f"{p}.self_attn_layer_scale.scale"] = ((HIDDEN,), "scale", 0.1)
        s[f"{p}.post_attention_layernorm.weight"] = ((HIDDEN,), "one", 0.0)
        s[f"{p}.mlp.gate_proj.weight"] = ((INTER, HIDDEN), "normal", 1 / math.sqrt(HIDDEN))
        s[f"{p}.mlp.up_proj.weight"] = ((INTER, HIDDEN), "normal", 1 / math.sqrt(HIDDEN))
        s[f"{p}.mlp.down_proj.weight"] = ((HIDDEN, INTER), "normal", 1 / math.sqrt(INTER))
        s[f"{p}.mlp_layer_scale.scale"] = ((HIDDEN,), "scale", 0.1)
    for i in range(2):
        p = f"decoder.upsample.{i}"
        s[f"{p}.0.conv.weight"] = ((UP_CH, UP_CH, 2), "normal", 1 / math.sqrt(UP_CH))
        s[f"{p}.0.conv.bias"] = ((UP_CH,), "normal", 0.02)
        s[f"{p}.1.dwconv.conv.weight"] = ((UP_CH, 1, 7), "normal", 1 / math.sqrt(7))
        s[f"{p}.1.dwconv.conv.bias"] = ((UP_CH,), "normal", 0.02)
        s[f"{p}.1.norm.weight"] = ((UP_CH,), "one", 0.0)
        s[f"{p}.1.norm.bias"] = ((UP_CH,), "zero", 0.0)
        s[f"{p}.1.pwconv1.weight"] = ((CONVNEXT_INTER, UP_CH), "normal", 1 / math.sqrt(UP_CH))
        s[f"{p}.1.pwconv1.bias"] = ((CONVNEXT_INTER,), "normal", 0.02)
        s[f"{p}.1.pwconv2.weight"] = ((UP_CH, CONVNEXT_INTER), "normal",
                                      1 / math.sqrt(CONVNEXT_INTER))
        s[f"{p}.1.pwconv2.bias"] = ((UP_CH,), "normal", 0.02)
        s[f"{p}.1.gamma"] = ((UP_CH,), "scale", 0.1)
    s["decoder.decoder.0.conv.weight"] = ((DECODER_INIT, PRE_CONV_OUT, 7), "normal",
                                          1 / math.sqrt(PRE_CONV_OUT * 7))
    s["decoder.decoder.0.conv.bias"] = ((DECODER_INIT,), "normal", 0.02)
    for b, (cin, cout, st) in enumerate(BLOCKS):
        p = f"decoder.decoder.{b + 1}.block"
        s[f"{p}.0.alpha"] = ((cin,), "log", 0.1)
        s[f"{p}.0.beta"] = ((cin,), "log", 0.1)
        s[f"{p}.1.conv.weight"] = ((cin, cout, 2 * st), "normal", 1 / math.sqrt(2 * cin))
        s[f"{p}.1.conv.bias"] = ((cout,), "normal", 0.02)
        for u in range(3):
            r = f"{p}.{u + 2}"
            s[f"{r}.act1.alpha"] = ((cout,), "log", 0.1)
            s[f"{r}.act1.beta"] = ((cout,), "log", 0.1)
            s[f"{r}.conv1.conv.weight"] = ((cout, cout, 7), "normal", 1 / math.sqrt(7 * cout))
            s[f"{r}.conv1.conv.bias"] = ((cout,), "normal", 0.02)
            s[f"{r}.act2.alpha"] = ((cout,), "log", 0.1)
            s[f"{r}.act2.beta"] = ((cout,), "log", 0.1)
            s[f"{r}.conv2.conv.weight"] = ((cout, cout, 1), "normal", 0.5 / math.sqrt(cout))
            s[f"{r}.conv2.conv.bias"] = ((cout,), "normal", 0.02)
    s["decoder.decoder.5.alpha"] = ((96,), "log", 0.1)
    s["decoder.decoder.5.beta"] = ((96,), "log", 0.1)
    s["decoder.decoder.6.conv.weight"] = ((1, 96, 7), "normal", 0.05 / math.sqrt(96 * 7))
    s["decoder.decoder.6.conv.bias"] = ((1,), "normal", 0.02)
    return s


def generate(seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    specs = tensor_specs()
    for name in sorted(specs):
        shape, kind, scale = specs[name]
        if kind == "one":
            v = np.ones(shape, np.float32)
        elif kind == "zero":
            v = np.zeros(shape, np.float32)
        elif kind == "usage":
            v = rng.uniform(0.5, 2.0, size=shape).astype(np.float32)
        elif kind == "scale":
            v = (np.float32(scale) + np.float32(0.01) *
                 rng.standard_normal(size=shape, dtype=np.float32)).astype(np.float32)
        else:  # normal / log
            v = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(scale)
        out[name] = np.ascontiguousarray(v, dtype=np.float32)
    return out


def write_f32_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    header: dict = {"__metadata__": {"format": "pt"}}
    offset = 0
    order = sorted(tensors)
    for name in order:
        n = tensors[name].size * 4
        header[name] = {"dtype": "F32", "shape": list(tensors[name].shape),
                        "data_offsets": [offset, offset + n]}
        offset += n
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for name in order:
            f.write(tensors[name].tobytes())


def write_codec(model_dir, seed: int = 0) -> dict[str, np.ndarray]:
    """Writes <model_dir>/speech_tokenizer/model.safetensors; returns the tensors."""
    t = generate(seed)
    p = Path(model_dir) / "speech_tokenizer" / "model.safetensors"
    if not p.exists():
        write_f32_safetensors(p, t)
    return t


class CodecOracle:
    """fp32 restatement of HipCodecInitial on the CPU (torch)."""

    def __init__(self, tensors: dict[str, np.ndarray]):
        import torch

        self.t = {k: torch.from_numpy(np.array(v, dtype=np.float32)) for k, v in tensors.items()}

    # ---- helpers (each cites the reference kernel it restates)
    @staticmethod
    def _causal_conv(x, w, b, dilation=1):
        """codec_causal_conv1d_dilated_f32 (kernels.rs:751-780): left pad d*(k-1)."""
        import torch.nn.functional as F

        k = w.shape[-1]
        x = F.pad(x, (dilation * (k - 1), 0))
        return F.conv1d(x[None], w, b, dilation=dilation)[0]

    @staticmethod
    def _transconv(x, w, b, stride):
        """codec_transconv1d_channels_f32 (kernels.rs:833-863): first in*stride samples."""
        import torch.nn.functional as F

        y = F.conv_transpose1d(x[None], w, b, stride=stride)[0]
        return y[:, : x.shape[1] * stride]

    @staticmethod
    def _snake(x, alpha, beta):
        """codec_snake_beta_f32 (kernels.rs:731-749)."""
        import torch

        a = torch.exp(alpha)[:, None]
        bb = torch.exp(beta)[:, None]
        s = torch.sin(x * a)
        return x + (s * s) / (bb + 1e-9)

    @staticmethod
    def _rms(x_tc, g, eps):
        """rmsnorm_f32 (kernels.rs:2-37) over the channel axis of [T, C]."""
        import torch

        return x_tc * torch.rsqrt((x_tc * x_tc).mean(-1, keepdim=True) + eps) * g

    @staticmethod
    def _rope(x_bhsd, theta):
        """rope_bhsd_f32 (kernels.rs:40-77): angle = t / theta^(2i/d), rotate-half."""
        import torch

        h, T, d = x_bhsd.shape
        half = d // 2
        i = torch.arange(half, dtype=torch.float32)
        expo = (i * 2) / float(d)
        t = torch.arange(T, dtype=torch.float32)[:, None]
        ang = t / torch.pow(torch.tensor(theta, dtype=torch.float32), expo)[None]
        c, s = torch.cos(ang), torch.sin(ang)
        a, b = x_bhsd[..., :half], x_bhsd[..., half:]
        return torch.cat([a * c - b * s, b * c + a * s], dim=-1)

    def rvq(self, codes: np.ndarray):
        """codec_rvq_project_f32 + load_normalized_codebook -> [512, T]."""
        import torch

        t = self.t
        codes = np.asarray(codes, dtype=np.int64).reshape(-1, GROUPS) % CODEBOOK_SIZE
        q = "decoder.quantizer"

        def book(name):
            e = t[f"{name}._codebook.embedding_sum"]
            u = torch.clamp(t[f"{name}._codebook.cluster_usage"], min=1e-7)
            return e / u[:, None]

        first = book(f"{q}.rvq_first.vq.layers.0")[torch.from_numpy(codes[:, 0])]
        rest = torch.zeros_like(first)
        for g in range(1, GROUPS):
            rest = rest + book(f"{q}.rvq_rest.vq.layers.{g - 1}")[torch.from_numpy(codes[:, g])]
        wf = t[f"{q}.rvq_first.output_proj.weight"][:, :, 0]
        wr = t[f"{q}.rvq_rest.output_proj.weight"][:, :, 0]
        return (first @ wf.T + rest @ wr.T).T.contiguous()

    def pre_transformer(self, x_ct):
        import torch

        t = self.t
        p = "decoder.pre_transformer"
        T = x_ct.shape[1]
        h = x_ct.T @ t[f"{p}.input_proj.weight"].T + t[f"{p}.input_proj.bias"]
        mask = torch.triu(torch.ones(T, T, dtype=torch.bool), diagonal=1)
        for i in range(LAYERS):
            L = f"{p}.layers.{i}"
            n = self._rms(h, t[f"{L}.input_layernorm.weight"], 1e-5)

            def heads(w):
                return (n @ w.T).reshape(T, HEADS, HEAD_DIM).permute(1, 0, 2)

            q = self._rope(heads(t[f"{L}.self_attn.q_proj.weight"]), 10000.0)
            k = self._rope(heads(t[f"{L}.self_attn.k_proj.weight"]), 10000.0)
            v = heads(t[f"{L}.self_attn.v_proj.weight"])
            sc = (q @ k.transpose(1, 2)) * (1.0 / math.sqrt(HEAD_DIM))
            sc = sc.masked_fill(mask, -3.4028234663852886e38)
            pr = torch.softmax(sc, dim=-1)
            att = (pr @ v).permute(1, 0, 2).reshape(T, HEADS * HEAD_DIM)
            h = h + (att @ t[f"{L}.self_attn.o_proj.weight"].T) * t[f"{L}.self_attn_layer_scale.scale"]
            n2 = self._rms(h, t[f"{L}.post_attention_layernorm.weight"], 1e-5)
            g = n2 @ t[f"{L}.mlp.gate_proj.weight"].T
            u = n2 @ t[f"{L}.mlp.up_proj.weight"].T
            m = (g / (1.0 + torch.exp(-g)) * u) @ t[f"{L}.mlp.down_proj.weight"].T
            h = h + m * t[f"{L}.mlp_layer_scale.scale"]
        n = self._rms(h, t[f"{p}.norm.weight"], 1e-5)
        out = n @ t[f"{p}.output_proj.weight"].T + t[f"{p}.output_proj.bias"]
        return out.T.contiguous()

    def upsample(self, x_ct):
        import torch
        import torch.nn.functional as F

        t = self.t
        for i in range(2):
            p = f"decoder.upsample.{i}"
            y = self._transconv(x_ct, t[f"{p}.0.conv.weight"], t[f"{p}.0.conv.bias"], 2)
            dw = F.conv1d(F.pad(y, (6, 0))[None], t[f"{p}.1.dwconv.conv.weight"],
                          t[f"{p}.1.dwconv.conv.bias"], groups=UP_CH)[0]
            z = dw.T
            mean = z.mean(-1, keepdim=True)
            var = torch.clamp((z * z).mean(-1, keepdim=True) - mean * mean, min=0.0)
            z = (z - mean) * torch.rsqrt(var + 1e-6) * t[f"{p}.1.norm.weight"] + t[f"{p}.1.norm.bias"]
            z = z @ t[f"{p}.1.pwconv1.weight"].T + t[f"{p}.1.pwconv1.bias"]
            z = 0.5 * z * (1.0 + torch.erf(z * 0.7071067811865476))
            z = z @ t[f"{p}.1.pwconv2.weight"].T + t[f"{p}.1.pwconv2.bias"]
            x_ct = y + z.T * t[f"{p}.1.gamma"][:, None]
        return x_ct

    def decoder(self, x_ct):
        import torch

        t = self.t
        x = self._causal_conv(x_ct, t["decoder.decoder.0.conv.weight"],
                              t["decoder.decoder.0.conv.bias"])
        for b, (_, _, st) in enumerate(BLOCKS):
            p = f"decoder.decoder.{b + 1}.block"
            x = self._snake(x, t[f"{p}.0.alpha"], t[f"{p}.0.beta"])
            x = self._transconv(x, t[f"{p}.1.conv.weight"], t[f"{p}.1.conv.bias"], st)
            for u, d in enumerate(DILATIONS):
                r = f"{p}.{u + 2}"
                y = self._snake(x, t[f"{r}.act1.alpha"], t[f"{r}.act1.beta"])
                y = self._causal_conv(y, t[f"{r}.conv1.conv.weight"], t[f"{r}.conv1.conv.bias"], d)
                y = self._snake(y, t[f"{r}.act2.alpha"], t[f"{r}.act2.beta"])
                y = self._causal_conv(y, t[f"{r}.conv2.conv.weight"], t[f"{r}.conv2.conv.bias"])
                x = x + y
        x = self._snake(x, t["decoder.decoder.5.alpha"], t["decoder.decoder.5.beta"])
        x = self._causal_conv(x, t["decoder.decoder.6.conv.weight"], t["decoder.decoder.6.conv.bias"])
        return torch.clamp(x[0], -1.0, 1.0)

    def decode(self, codes) -> np.ndarray:
        """HipTtsEngine::decode_codes (generation.rs:619-646): codes [frames*16] -> samples."""
        import torch

        codes = np.asarray(codes, dtype=np.int64).reshape(-1)
        if codes.size == 0:
            return np.zeros(0, np.float32)
        with torch.inference_mode():
            x = self.rvq(codes)
            x = self._causal_conv(x, self.t["decoder.pre_conv.conv.weight"],
                                  self.t["decoder.pre_conv.conv.bias"])
            x = self.pre_transformer(x)
            x = self.upsample(x)
            return self.decoder(x).numpy().astype(np.float32)

    def decode_stages(self, codes) -> dict[str, np.ndarray]:
        """Intermediate tensors for stage-by-stage parity (channel-major)."""
        import torch

        codes = np.asarray(codes, dtype=np.int64).reshape(-1)
        with torch.inference_mode():
            out = {}
            x = self.rvq(codes)
            out["rvq"] = x.numpy().copy()
            x = self._causal_conv(x, self.t["decoder.pre_conv.conv.weight"],
                                  self.t["decoder.pre_conv.conv.bias"])
            out["pre_conv"] = x.numpy().copy()
            x = self.pre_transformer(x)
            out["pre_transformer"] = x.numpy().copy()
            x = self.upsample(x)
            out["upsample"] = x.numpy().copy()
            out["waveform"] = self.decoder(x).numpy().copy()
        return out
