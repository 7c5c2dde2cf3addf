"""CPU fp32 restatement of the reference Qwen3-TTS token loop (the parity oracle).

TEST INFRASTRUCTURE ONLY: tests, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg use this module as the checker; the product path never imports
it.

It restates, in PyTorch-CPU float32, what ``piedshag/qwen3-tts-hip`` computes
for the talker decode step and the CodePredictor pass (each function cites the
reference file:line it follows):

* prefill rows from content ids           -- src/model/text.rs:516-603
* decoder layer, prefill (causal, offset 0) -- src/model/decode.rs:1077-1298
* decoder layer, decode at a cache offset  -- src/model/decode.rs:1694-1894
* RMSNorm / RoPE / softmax / argmax kernels -- src/gpu/kernels.rs:2-76,121-220
* GQA mapping, 1/sqrt(d) scale            -- src/gpu/kernels.rs:1048-1119
* talker head, penalty, suppression        -- src/model/talker.rs:431-496,
                                              src/gpu/kernels.rs:248-263,408-426
* device top-k sampler                     -- src/gpu/kernels.rs:265-406
* CPU sampler + LCG                        -- src/model/sampling.rs:40-126
* CodePredictor pass                       -- src/model/code_predictor.rs:366-471,754-862
* rollout loop / streams                   -- src/generation.rs:657-749,876-963

Parity to the reference's own Python oracle (the external ``qwen_tts``
package) is not pinned here: that package and the real checkpoints are absent.
The restatement follows the Rust reference, which is the executable spec.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from . import synth

F32_MAX = np.float32(3.4028234663852886e38)
LCG_MUL = 6364136223846793005
LCG_INC = 1442695040888963407
MASK64 = (1 << 64) - 1
SEED_XOR = 0x9E3779B97F4A7C15
NEWLINE = 198  # src/model/text.rs:15


# ----------------------------------------------------------------------------
# sampling (src/model/sampling.rs)
# ----------------------------------------------------------------------------
@dataclass(frozen=True)
class SamplingConfig:
    do_sample: bool
    top_k: int
    top_p: float
    temperature: float

    def supports_device_sampling(self) -> bool:
        """sampling.rs:28-37 (the env override is not modelled)."""
        return self.do_sample and 0 < self.top_k <= 256 and self.top_p >= 0.999999


class Lcg:
    """64-bit LCG, top 24 bits / 2^24 (sampling.rs:120-126)."""

    def __init__(self, seed: int):
        self.state = (seed ^ SEED_XOR) & MASK64

    def next_f32(self) -> np.float32:
        self.state = (self.state * LCG_MUL + LCG_INC) & MASK64
        bits = self.state >> 40
        return np.float32(bits) / np.float32(1 << 24)


def philox_uniform(seed: int, counter: int) -> np.float32:
    """Philox-4x32-10 (Salmon et al. 2011) on (counter, 0) with key = seed; the
    first output word's top 24 bits / 2^24. Used only in the Philox RNG mode,
    which has no reference counterpart (the reference draws from the LCG)."""
    M0, M1 = 0xD2511F53, 0xCD9E8D57
    W0, W1 = 0x9E3779B9, 0xBB67AE85
    c0, c1, c2, c3 = counter & 0xFFFFFFFF, (counter >> 32) & 0xFFFFFFFF, 0, 0
    k0, k1 = seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF
    for _ in range(10):
        p0 = M0 * c0
        p1 = M1 * c2
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return np.float32(c0 >> 8) / np.float32(1 << 24)


class PhiloxStream:
    def __init__(self, seed: int):
        self.seed = seed & MASK64
        self.counter = 0

    def next_f32(self) -> np.float32:
        u = philox_uniform(self.seed, self.counter)
        self.counter += 1
        return u


def argmax_device(logits: np.ndarray) -> int:
    """argmax_rows_f32 (kernels.rs:177-220): start at -FLT_MAX, lowest index wins ties."""
    best_v, best_i = -F32_MAX, 0
    v = logits.astype(np.float32)
    m = np.max(np.where(np.isnan(v), -np.inf, v))
    if m > best_v:
        best_i = int(np.flatnonzero(v == m)[0])
    return best_i


def _order_margin(vals, j: int) -> float:
    """Half the logit gap between the drawn candidate j and its neighbours in
    the sorted order: a logit error of that size can swap j with a neighbour,
    which hands j's bucket of the CDF to the other token."""
    best = float("inf")
    v = np.asarray(vals, dtype=np.float64)
    if j > 0:
        best = min(best, (v[j - 1] - v[j]) / 2.0)
    if j + 1 < v.size:
        best = min(best, (v[j] - v[j + 1]) / 2.0)
    return best


def _cdf_margin(probs, j: int, target0, temperature: float) -> float:
    """How robust an inverse-CDF draw is, in logit units: the smallest logit
    error that could move an edge of the drawn bucket j past the target.
    With every logit off by at most d, each probability exp((l - max) / T)
    moves by a factor of at most exp(2 d / T) (l and the max both move), and
    so do the mass C_e below an edge e and the target u * sum; the edge
    crosses the target only once 2 d / T >= |target - C_e| / (target + C_e).
    Sums in fp32, candidate order."""
    before = np.float32(0.0)
    for i in range(j):
        before = np.float32(before + probs[i])
    after = np.float32(before + probs[j])
    t = float(target0)
    best = float("inf")
    for edge in (float(before), float(after)):
        if t + edge > 0:
            best = min(best, abs(t - edge) / (t + edge) * float(temperature) / 2.0)
    return best


def sample_topk_device(logits: np.ndarray, top_k: int, temperature: float, u: np.float32,
                       with_margin: bool = False):
    """sample_topk_f32 (kernels.rs:265-336): non-finite -> -FLT_MAX, sort descending,
    softmax over the first min(top_k, vocab) entries in fp32, inverse CDF on u*sum.
    Ties are ordered by lowest index (the reference's bitonic order for exact ties
    is unspecified; finite random logits do not tie)."""
    v = np.where(np.isfinite(logits), logits, -F32_MAX).astype(np.float32)
    order = np.lexsort((np.arange(v.size), -v.astype(np.float64)))
    vals = v[order]
    kept = min(top_k, v.size)
    mx = vals[0]
    t = np.float32(temperature)
    probs = np.empty(kept, dtype=np.float32)
    s = np.float32(0.0)
    for i in range(kept):
        p = np.float32(math.exp(np.float32(np.float32(vals[i] - mx) / t)))
        probs[i] = p
        s = np.float32(s + p)
    if not np.isfinite(s) or s <= 0:
        return (int(order[0]), float("inf")) if with_margin else int(order[0])
    target = np.float32(np.float32(u) * s)
    target0, pick = target, kept - 1
    for i in range(kept):
        if target <= probs[i]:
            pick = i
            break
        target = np.float32(target - probs[i])
    tok = int(order[pick])
    if not with_margin:
        return tok
    # neighbours include the first candidate past top_k (a swap there changes
    # the candidate set when the draw is the last bucket)
    return tok, min(_cdf_margin(probs, pick, target0, temperature),
                    _order_margin(vals[: kept + 1], pick))


def sample_cpu(logits: np.ndarray, cfg: SamplingConfig, rng, with_margin: bool = False):
    """sampling.rs:53-118: finite candidates, stable descending sort, top-k,
    softmax((l-max)/T), optional top-p renormalisation, inverse CDF on u.
    No draw when the probability sum is not finite/positive (sampling.rs:79-81)."""
    idx = np.flatnonzero(np.isfinite(logits))
    if idx.size == 0:
        raise ValueError("cannot sample from logits with no finite values")
    vals = logits[idx].astype(np.float32)
    order = np.lexsort((idx, -vals.astype(np.float64)))  # stable: ties keep index order
    idx, vals = idx[order], vals[order]
    sorted_vals = vals
    if 0 < cfg.top_k < idx.size:
        idx, vals = idx[: cfg.top_k], vals[: cfg.top_k]
    mx = vals[0]
    t = np.float32(cfg.temperature)
    probs = np.array([np.float32(math.exp(np.float32(np.float32(x - mx) / t))) for x in vals],
                     dtype=np.float32)
    s = np.float32(0)
    for p in probs:
        s = np.float32(s + p)
    if not np.isfinite(s) or s <= 0:
        return (int(idx[0]), float("inf")) if with_margin else int(idx[0])
    probs = (probs / s).astype(np.float32)
    if cfg.top_p < 1.0:
        cum, keep = np.float32(0), 0
        for p in probs:
            keep += 1
            cum = np.float32(cum + p)
            if cum >= np.float32(cfg.top_p):
                break
        keep = max(keep, 1)
        idx, probs = idx[:keep], probs[:keep]
        ks = np.float32(0)
        for p in probs:
            ks = np.float32(ks + p)
        if ks > 0:
            probs = (probs / ks).astype(np.float32)
    target = rng.next_f32()
    target0, pick = target, len(idx) - 1
    for i, p in enumerate(probs):
        if target <= p:
            pick = i
            break
        target = np.float32(target - p)
    tok = int(idx[pick])
    if not with_margin:
        return tok
    return tok, min(_cdf_margin(probs, pick, target0, cfg.temperature),
                    _order_margin(sorted_vals[: len(idx) + 1], pick))


def select(logits: np.ndarray, cfg: SamplingConfig, rng) -> int:
    """Token selection as the reference engine routes it: greedy -> device argmax;
    device-eligible -> one draw + device top-k; else CPU sampler."""
    return select_margin(logits, cfg, rng)[0]


def select_margin(logits: np.ndarray, cfg: SamplingConfig, rng):
    """select() plus how robust its choice is against small logit errors:
    greedy -> the top-2 logit gap; sampled -> the smallest logit error that
    could move an edge of the drawn bucket past the inverse-CDF target (both
    in logit units).
    A GPU run whose logits differ from these by bf16 rounding can pick a
    different token only where this margin is small."""
    if not cfg.do_sample:
        return argmax_device(logits), top2_gap(logits)
    if cfg.supports_device_sampling():
        u = rng.next_f32()
        return sample_topk_device(logits, cfg.top_k, cfg.temperature, u, with_margin=True)
    return sample_cpu(logits, cfg, rng, with_margin=True)


def top2_gap(logits: np.ndarray) -> float:
    v = np.sort(logits[np.isfinite(logits)].astype(np.float64))
    return float(v[-1] - v[-2]) if v.size >= 2 else float("inf")


# ----------------------------------------------------------------------------
# kernels (src/gpu/kernels.rs)
# ----------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    """rmsnorm_f32 (kernels.rs:2-37): x * rsqrt(mean(x^2) + eps) * gamma per row."""
    inv = torch.rsqrt((x * x).sum(-1, keepdim=True) / x.shape[-1] + eps)
    return x * inv * gamma


def rope_tables(theta: float, head_dim: int, positions: np.ndarray):
    """Angle = pos / powf(theta, 2i/d) in fp32 (kernels.rs:64-67)."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    exponent = (i * np.float32(2)) / np.float32(head_dim)
    denom = np.power(np.float32(theta), exponent, dtype=np.float32)
    ang = positions.astype(np.float32)[:, None] / denom[None, :]
    return torch.from_numpy(np.cos(ang).astype(np.float32)), torch.from_numpy(
        np.sin(ang).astype(np.float32))


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rotate-half RoPE (kernels.rs:41-76). x: [steps, heads, d]; cos/sin: [steps, d/2]."""
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat((a * c - b * s, b * c + a * s), dim=-1)


# ----------------------------------------------------------------------------
# model
# ----------------------------------------------------------------------------
@dataclass
class StackDims:
    hidden: int
    intermediate: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    eps: float
    theta: float


class DecoderStack:
    """DecodeStepStack (decode.rs): N Qwen3 decoder layers with an fp32 KV cache
    [kv_heads, max_steps, head_dim] per layer (decode.rs:1897-1905)."""

    def __init__(self, w: dict, prefix: str, dims: StackDims, max_steps: int):
        self.d = dims
        self.max_steps = max_steps
        self.layers = []
        for i in range(dims.layers):
            p = f"{prefix}.{i}"
            g = lambda n: torch.from_numpy(np.ascontiguousarray(w[f"{p}.{n}"], dtype=np.float32))
            self.layers.append({
                "in_g": g("input_layernorm.weight"), "q_g": g("self_attn.q_norm.weight"),
                "k_g": g("self_attn.k_norm.weight"), "q": g("self_attn.q_proj.weight"),
                "k": g("self_attn.k_proj.weight"), "v": g("self_attn.v_proj.weight"),
                "o": g("self_attn.o_proj.weight"), "post_g": g("post_attention_layernorm.weight"),
                "gate": g("mlp.gate_proj.weight"), "up": g("mlp.up_proj.weight"),
                "down": g("mlp.down_proj.weight"),
            })
        self.reset()

    def reset(self):
        d = self.d
        self.k_cache = [torch.zeros(d.kv_heads, self.max_steps, d.head_dim) for _ in self.layers]
        self.v_cache = [torch.zeros(d.kv_heads, self.max_steps, d.head_dim) for _ in self.layers]

    def _layer(self, li: int, x: torch.Tensor, offset: int) -> torch.Tensor:
        """One layer on rows x [S, H] at cache positions offset..offset+S-1.
        With offset 0 this is prefill_forward (decode.rs:1077-1298); with S=1 it is
        decode_step_layer (decode.rs:1694-1894). Causal: key <= offset + query."""
        d, L = self.d, self.layers[li]
        S = x.shape[0]
        normed = rmsnorm(x, L["in_g"], d.eps)
        q = (normed @ L["q"].T).view(S, d.q_heads, d.head_dim)
        k = (normed @ L["k"].T).view(S, d.kv_heads, d.head_dim)
        v = (normed @ L["v"].T).view(S, d.kv_heads, d.head_dim)
        q = rmsnorm(q, L["q_g"], d.eps)
        k = rmsnorm(k, L["k_g"], d.eps)
        cos, sin = rope_tables(d.theta, d.head_dim, np.arange(offset, offset + S))
        q = rope(q, cos, sin)
        k = rope(k, cos, sin)
        self.k_cache[li][:, offset:offset + S] = k.transpose(0, 1)
        self.v_cache[li][:, offset:offset + S] = v.transpose(0, 1)
        T = offset + S
        kc = self.k_cache[li][:, :T]  # [kvh, T, d]
        vc = self.v_cache[li][:, :T]
        group = d.q_heads // d.kv_heads
        kv_of_q = torch.arange(d.q_heads) // group  # kernels.rs:1028,1067
        scale = np.float32(1.0 / math.sqrt(d.head_dim))
        scores = torch.einsum("shd,htd->hst", q, kc[kv_of_q]) * scale
        qpos = torch.arange(offset, offset + S)[:, None]
        kpos = torch.arange(T)[None, :]
        scores = scores.masked_fill((kpos > qpos)[None], -float(F32_MAX))
        probs = torch.softmax(scores, dim=-1)
        att = torch.einsum("hst,htd->shd", probs, vc[kv_of_q]).reshape(S, -1)
        h1 = x + att @ L["o"].T
        post = rmsnorm(h1, L["post_g"], d.eps)
        gate = post @ L["gate"].T
        up = post @ L["up"].T
        act = gate / (1.0 + torch.exp(-gate)) * up  # swiglu_f32 (kernels.rs:106-117)
        return h1 + act @ L["down"].T

    def forward(self, x: torch.Tensor, offset: int) -> torch.Tensor:
        if offset + x.shape[0] > self.max_steps:
            raise ValueError("offset outside cache")
        for li in range(len(self.layers)):
            x = self._layer(li, x, offset)
        return x


@dataclass
class FrameRecord:
    semantic: int
    talker_gap: float
    acoustic: list
    cp_gaps: list
    # select_margin() of each token: the semantic token, then the 15 acoustic
    # tokens (equal to the gaps for greedy selection)
    talker_margin: float = float("inf")
    cp_margins: list = field(default_factory=list)


class OracleModel:
    """Talker + CodePredictor + text prep on synthetic (or real) safetensors."""

    def __init__(self, model_dir, max_cache_steps: int = 512):
        model_dir = Path(model_dir)
        cfg = json.loads((model_dir / "config.json").read_text())
        self.cfg = cfg
        t = cfg["talker_config"]
        cp = t["code_predictor_config"]
        w = synth.read_safetensors(model_dir / "model.safetensors")
        self.tdims = StackDims(t["hidden_size"], t["intermediate_size"], t["num_hidden_layers"],
                               t["num_attention_heads"], t["num_key_value_heads"], t["head_dim"],
                               t["rms_norm_eps"], t["rope_theta"])
        self.cdims = StackDims(cp["hidden_size"], cp["intermediate_size"], cp["num_hidden_layers"],
                               cp["num_attention_heads"], cp["num_key_value_heads"], cp["head_dim"],
                               cp["rms_norm_eps"], cp["rope_theta"])
        self.vocab = t["vocab_size"]
        self.cp_vocab = cp["vocab_size"]
        self.groups = t["num_code_groups"]
        self.codec_eos = t["codec_eos_token_id"]
        self.talker = DecoderStack(w, "talker.model.layers", self.tdims, max_cache_steps)
        self.cp = DecoderStack(w, "talker.code_predictor.model.layers", self.cdims,
                               cp["num_code_groups"])
        T = lambda n: torch.from_numpy(np.ascontiguousarray(w[n], dtype=np.float32))
        self.norm = T("talker.model.norm.weight")
        self.head = T("talker.codec_head.weight")
        self.codec_emb = T("talker.model.codec_embedding.weight")
        self.cp_norm = T("talker.code_predictor.model.norm.weight")
        self.lm_heads = [T(f"talker.code_predictor.lm_head.{g}.weight")
                         for g in range(self.groups - 1)]
        self.cp_embs = [T(f"talker.code_predictor.model.codec_embedding.{g}.weight")
                        for g in range(self.groups - 1)]
        self.proj_w = self.proj_b = None
        if self.cdims.hidden != self.tdims.hidden:
            self.proj_w = T("talker.code_predictor.small_to_mtp_projection.weight")
            self.proj_b = T("talker.code_predictor.small_to_mtp_projection.bias")
        self.text_emb = w["talker.model.text_embedding.weight"]  # numpy (large)
        self.fc1_w = T("talker.text_projection.linear_fc1.weight")
        self.fc1_b = T("talker.text_projection.linear_fc1.bias")
        self.fc2_w = T("talker.text_projection.linear_fc2.weight")
        self.fc2_b = T("talker.text_projection.linear_fc2.bias")

    # ---- text prep (text.rs:516-603) -------------------------------------
    def projected_text(self, ids) -> torch.Tensor:
        """fc2(silu(fc1(emb[id]))) per token (text.rs:571-602, 700-716)."""
        e = torch.from_numpy(np.ascontiguousarray(self.text_emb[np.asarray(ids, dtype=np.int64)],
                                                  dtype=np.float32))
        h = e @ self.fc1_w.T + self.fc1_b
        h = h / (1.0 + torch.exp(-h))
        return h @ self.fc2_w.T + self.fc2_b

    def codec_rows(self, ids) -> torch.Tensor:
        return self.codec_emb[torch.as_tensor(ids, dtype=torch.long)]

    def build_prefill(self, text_ids, speaker="ryan", language="english") -> torch.Tensor:
        """build_prefill_with_speaker_embedding (text.rs:530-569): 3 role rows,
        6 tts+codec rows, then one text+codec row per lookahead token."""
        c, t = self.cfg, self.cfg["talker_config"]
        spk = t["spk_id"][speaker]
        lang = t["codec_language_id"][language]
        role = self.projected_text([c["im_start_token_id"], c["assistant_token_id"], NEWLINE])
        codec_prefix = self.codec_rows([t["codec_think_id"], t["codec_think_bos_id"], lang,
                                        t["codec_think_eos_id"], t["codec_pad_id"],
                                        t["codec_bos_id"]])
        codec = torch.cat([codec_prefix[:4], self.codec_rows([spk]), codec_prefix[4:]])
        pad, bos = c["tts_pad_token_id"], c["tts_bos_token_id"]
        tts = self.projected_text([pad, pad, pad, pad, pad, bos])
        rows = [role, tts + codec[:6]]
        if len(text_ids):
            text = self.projected_text(text_ids)
            ci = torch.full((len(text_ids),), 5, dtype=torch.long)
            ci[-1] = 6
            rows.append(text + codec[ci])
        return torch.cat(rows)

    def prepare(self, content_ids, lookahead=None, speaker="ryan", language="english"):
        """prepare_custom_voice_with_lookahead (text.rs:348-382) from content ids:
        lookahead None means all content in the prefill (generation.rs:360-366)."""
        n = len(content_ids)
        la = 0 if n == 0 else (n if lookahead is None else max(1, min(lookahead, n)))
        prefill = self.build_prefill(list(content_ids[:la]), speaker, language)
        trailing_ids = list(content_ids[la:]) + [self.cfg["tts_eos_token_id"]]
        trailing = self.projected_text(trailing_ids)
        pad = self.projected_text([self.cfg["tts_pad_token_id"]])[0]
        return prefill, trailing, pad

    # ---- talker (talker.rs) ----------------------------------------------
    def talker_logits(self, pre_norm: torch.Tensor):
        """final RMSNorm -> codec_head (talker.rs:438-453)."""
        hidden = rmsnorm(pre_norm, self.norm, self.tdims.eps)
        return hidden, hidden @ self.head.T

    def penalise_and_suppress(self, logits: np.ndarray, history, penalty: float) -> np.ndarray:
        """apply_repetition_penalty_f32 per occurrence (kernels.rs:408-426), then
        suppress_codec_logits_f32 (kernels.rs:248-263)."""
        out = logits.astype(np.float32).copy()
        if history is not None and len(history) and penalty != 1.0:
            p = np.float32(penalty)
            for tok in history:
                if 0 <= tok < out.size:
                    v = out[tok]
                    out[tok] = np.float32(v * p) if v < 0 else np.float32(v / p)
        out[self.vocab - 1024:] = np.where(np.arange(self.vocab - 1024, self.vocab)
                                           == self.codec_eos, out[self.vocab - 1024:], -np.inf)
        return out

    def talker_prefill(self, rows: torch.Tensor):
        self.talker.reset()
        out = self.talker.forward(rows, 0)
        hidden, logits = self.talker_logits(out[-1])
        return out[-1], hidden, logits.numpy()

    def talker_step(self, step_input: torch.Tensor, pos: int):
        out = self.talker.forward(step_input[None], pos)[0]
        hidden, logits = self.talker_logits(out)
        return out, hidden, logits.numpy()

    # ---- CodePredictor (code_predictor.rs) --------------------------------
    def project(self, x: torch.Tensor) -> torch.Tensor:
        """project_to_stack (code_predictor.rs:754-787)."""
        if self.proj_w is None:
            return x
        return x @ self.proj_w.T + self.proj_b

    def cp_logits(self, h: torch.Tensor, g: int) -> np.ndarray:
        """logits_for_hidden (code_predictor.rs:819-837)."""
        return (rmsnorm(h, self.cp_norm, self.cdims.eps) @ self.lm_heads[g].T).numpy()

    def code_predictor(self, talker_hidden, semantic_embed, cfg: SamplingConfig, rng,
                       forced=None):
        """generate_inner[_sampled] (code_predictor.rs:366-471): 2-row prefill at
        positions 0,1, head 0, then groups g=1..14 decoded at offset g+1.
        ``forced`` (15 ids) replays given tokens (teacher forcing) while still
        consuming the same RNG draws, so logits can be compared along a path.
        Returns the path's tokens; the oracle's own choice at every step (what
        it would have selected on that path) is kept in ``last_cp_choices``."""
        self.cp.reset()
        prefix = torch.stack([talker_hidden, semantic_embed])
        out = self.cp.forward(self.project(prefix), 0)
        tokens, gaps, all_logits, margins, choices = [], [], [], [], []
        h = out[1]
        emb_sum = None
        for g in range(self.groups - 1):
            if g > 0:
                h = self.cp.forward(self.project(cur)[None], g + 1)[0]
            lg = self.cp_logits(h, g)
            all_logits.append(lg)
            gaps.append(top2_gap(lg))
            tok, margin = select_margin(lg, cfg, rng)
            margins.append(margin)
            choices.append(tok)
            if forced is not None:
                tok = int(forced[g])
            tokens.append(tok)
            cur = self.cp_embs[g][tok]
            emb_sum = cur.clone() if emb_sum is None else emb_sum + cur
        self.last_cp_margins = margins
        self.last_cp_choices = choices
        return tokens, emb_sum, gaps, all_logits

    # ---- rollout (generation.rs:657-749) ----------------------------------
    def rollout(self, prefill, trailing, tts_pad, max_frames: int, talker_cfg: SamplingConfig,
                sub_cfg: SamplingConfig, penalty: float = 1.0, seed: int = 0, rng_kind="lcg",
                forced_codes=None):
        """Frame loop: EOS check, CP prefix, CP pass, append 16 codes, step input,
        talker decode at P+frame. ``forced_codes`` ([frames*16]) teacher-forces
        the path so per-frame choices can be checked against another run: the
        returned codes are then the ORACLE'S OWN choices at every step of the
        forced path (not the forced codes), frame count and EOS follow the
        path, and ``final_choice`` / ``final_margin`` hold the oracle's choice
        (and its margin) for the semantic token that ended the path (None when
        max_frames ended it)."""
        rng = Lcg(seed) if rng_kind == "lcg" else PhiloxStream(seed)
        P = prefill.shape[0]
        _, hidden, logits = self.talker_prefill(prefill)
        logits = self.penalise_and_suppress(logits, None, 1.0)
        semantic, margin = select_margin(logits, talker_cfg, rng)
        choice = semantic
        gaps = [top2_gap(logits)]
        margins = [margin]
        if forced_codes is not None and len(forced_codes) >= 16:
            semantic = int(forced_codes[0])
        elif forced_codes is not None:
            semantic = self.codec_eos  # the forced path produced no frame: it ended here
        codes, history, records = [], [], []
        ended = False
        self.final_choice, self.final_margin = None, None
        for frame in range(max_frames):
            if semantic == self.codec_eos:
                ended = True
                self.final_choice, self.final_margin = choice, margins[-1]
                break
            sem_emb = self.codec_emb[semantic]
            forced = None
            if forced_codes is not None and len(forced_codes) >= 16 * (frame + 1):
                forced = forced_codes[16 * frame + 1: 16 * frame + 16]
            toks, emb_sum, cp_gaps, _ = self.code_predictor(hidden, sem_emb, sub_cfg, rng, forced)
            codes.append(choice)
            codes.extend(self.last_cp_choices)
            history.append(semantic)
            records.append(FrameRecord(semantic, gaps[-1], toks, cp_gaps, margins[-1],
                                       list(self.last_cp_margins)))
            if frame + 1 < max_frames:
                tr = trailing[frame] if frame < trailing.shape[0] else tts_pad
                step = sem_emb + emb_sum + tr
                _, hidden, logits = self.talker_step(step, P + frame)
                use_hist = penalty != 1.0 or talker_cfg.do_sample
                logits = self.penalise_and_suppress(logits, history if use_hist else None, penalty)
                semantic, margin = select_margin(logits, talker_cfg, rng)
                choice = semantic
                gaps.append(top2_gap(logits))
                margins.append(margin)
                if forced_codes is not None and len(forced_codes) >= 16 * (frame + 2):
                    semantic = int(forced_codes[16 * (frame + 1)])
                elif forced_codes is not None:
                    semantic = self.codec_eos  # the forced path ended after this frame
        return codes, ended, records


def deterministic_hidden(length: int, modulus: int, center: float) -> np.ndarray:
    """((i % m) - c) / m, the CodePredictor parity inputs of the reference's
    python-reference/qwen3_tts_reference.py:620-626."""
    return np.array([((i % modulus) - center) / modulus for i in range(length)], dtype=np.float32)
