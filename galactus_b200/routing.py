"""Seeded synthetic router outputs for the MoE benchmarks (the router itself is
upstream of the routed-expert FFN; its outputs are this path's inputs).

Per layer and token: logits z_e + b_e with z ~ N(0,1) and a fixed per-expert
bias b_e = log of the Zipf(s) weight of the expert's rank (ranks permuted per
layer), optionally AR(1)-correlated across consecutive tokens
(z_t = rho z_{t-1} + sqrt(1 - rho^2) eps_t). Selection and weights follow the
model family:
  softmax_topk      softmax over all experts, top-k, weights = probabilities (OLMoE)
  softmax_topk_norm the same, weights renormalised over the k (Qwen3-MoE)
  topk_softmax      top-k logits, softmax over the k (gpt-oss)
  sigmoid_group     sigmoid scores, 8 groups, top-4 groups by their two best
                    scores, top-k inside them, normalised and scaled by 2.5
                    (DeepSeek-V3)
"""
from __future__ import annotations

import numpy as np

SCHEMES = {
    "olmoe-1b-7b": "softmax_topk",
    "qwen3-30b-a3b": "softmax_topk_norm",
    "gpt-oss-120b": "topk_softmax",
    "qwen3-235b-a22b": "softmax_topk_norm",
    "deepseek-v3": "sigmoid_group",
}


def zipf_bias(rng: np.random.Generator, experts: int, s: float = 1.1) -> np.ndarray:
    w = 1.0 / np.arange(1, experts + 1, dtype=np.float64) ** s
    w /= w.sum()
    return np.log(w)[rng.permutation(experts)]


def logits(model, tokens: int, layers: int, seed: int, rho: float = 0.0, s: float = 1.1) -> np.ndarray:
    """Router logits float32 [tokens, layers, E]: z + b with the Zipf rank bias
    and the AR(1) noise described above (the same stream as routes())."""
    rng = np.random.default_rng(seed)
    E = model.experts
    bias = np.stack([zipf_bias(rng, E, s) for _ in range(layers)])          # [layers, E]
    z = rng.standard_normal((layers, E))
    out = np.zeros((tokens, layers, E), np.float32)
    c = np.sqrt(1.0 - rho * rho)
    for t in range(tokens):
        if t > 0:
            z = rho * z + c * rng.standard_normal((layers, E))
        out[t] = z + bias
    return out


def routes(model, tokens: int, layers: int, seed: int, rho: float = 0.0, s: float = 1.1,
           scheme: str | None = None) -> tuple[np.ndarray, np.ndarray]:
    """ids int32 [tokens, layers, k], weights float32 [tokens, layers, k]."""
    scheme = scheme or SCHEMES.get(model.name, "softmax_topk_norm")
    rng = np.random.default_rng(seed)
    E, k = model.experts, model.used
    bias = np.stack([zipf_bias(rng, E, s) for _ in range(layers)])          # [layers, E]
    z = rng.standard_normal((layers, E))
    ids = np.zeros((tokens, layers, k), np.int32)
    wts = np.zeros((tokens, layers, k), np.float32)
    c = np.sqrt(1.0 - rho * rho)
    for t in range(tokens):
        if t > 0:
            z = rho * z + c * rng.standard_normal((layers, E))
        logits = z + bias
        if scheme == "sigmoid_group":
            score = 1.0 / (1.0 + np.exp(-logits))
            g = score.reshape(layers, 8, E // 8)
            gscore = np.sort(g, axis=2)[:, :, -2:].sum(axis=2)                  # [layers, 8]
            keep = np.argsort(-gscore, axis=1, kind="stable")[:, :4]
            mask = np.zeros((layers, 8), bool)
            np.put_along_axis(mask, keep, True, axis=1)
            masked = np.where(np.repeat(mask, E // 8, axis=1), score, -np.inf)
            sel = np.argsort(-masked, axis=1, kind="stable")[:, :k]
            w = np.take_along_axis(score, sel, axis=1)
            w = w / w.sum(axis=1, keepdims=True) * 2.5
        else:
            sel = np.argsort(-logits, axis=1, kind="stable")[:, :k]
            if scheme == "topk_softmax":
                lg = np.take_along_axis(logits, sel, axis=1)
                w = np.exp(lg - lg.max(axis=1, keepdims=True))
                w /= w.sum(axis=1, keepdims=True)
            else:
                p = np.exp(logits - logits.max(axis=1, keepdims=True))
                p /= p.sum(axis=1, keepdims=True)
                w = np.take_along_axis(p, sel, axis=1)
                if scheme == "softmax_topk_norm":
                    w = w / w.sum(axis=1, keepdims=True)
        ids[t] = sel
        wts[t] = w
    return ids, wts
