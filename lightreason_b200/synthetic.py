"""Seeded synthetic weights and inputs for the MoE layer of Qwen3.6-35B-A3B.

There is no checkpoint here, so every benchmark and test draws the layer from
fixed seeds with the shapes and value distributions of the reference's
benchmark configurations:

* hidden states ~ N(0, 1) in BF16;
* router W [256, 2048], expert gate_up [256, 1024, 2048] and down
  [256, 2048, 512], shared expert gate/up [512, 2048] and down [2048, 512], and
  the shared-expert gate [2048]: all ~ N(0, 0.02) in BF16 (the synthetic weights
  of edge35b/probe_experts.py:66-69 use the same std);
* a per-expert FP32 logit bias added before the router softmax, either
  ~ N(0, 0.5) ("normal") or alpha * ln p_pi(e) with p_k ~ k^-1.1 ("zipf"), which
  skews expert popularity like a Zipf(1.1) law.

Each tensor (and each expert of the expert banks) has its own numpy
SeedSequence, so a checker can draw only the experts a route needs.  numpy's
PCG64 and ziggurat normal are platform independent, so a seed yields the same
bits on every machine with the same numpy.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

HIDDEN = 2048
INNER = 512
SHARED_INNER = 512
EXPERTS = 256
TOP_K = 8
WEIGHT_STD = 0.02
# alpha for the Zipf(1.1) bias; frozen after a bisection that matched realised
# top-1 expert frequencies to k^-1.1 on N(0,1) activations (synthetic.py
# calibrate_zipf_alpha reproduces it).
ZIPF_S = 1.1
ZIPF_ALPHA = 0.4485

_TENSOR_IDS = {"router": 1, "bias": 2, "gate_up": 3, "down": 4, "sh_gate": 5, "sh_up": 6, "sh_down": 7,
               "sh_gate_w": 8, "x": 9, "perm": 10}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns (uint16), via torch's
    (multi-threaded, RNE) conversion."""
    import torch

    x = np.ascontiguousarray(x, dtype=np.float32)
    return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _rng(seed: int, *key: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([int(seed), *map(int, key)]))


def normal_bf16(seed: int, key: tuple, shape, std: float) -> np.ndarray:
    values = _rng(seed, *key).standard_normal(int(np.prod(shape)), dtype=np.float32)
    if std != 1.0:
        values *= np.float32(std)
    return f32_to_bf16_bits(values).reshape(shape)


def expert_gate_up(seed: int, layer: int, expert: int, hidden=HIDDEN, inner=INNER) -> np.ndarray:
    return normal_bf16(seed, (layer, _TENSOR_IDS["gate_up"], expert), (2 * inner, hidden), WEIGHT_STD)


def expert_down(seed: int, layer: int, expert: int, hidden=HIDDEN, inner=INNER) -> np.ndarray:
    return normal_bf16(seed, (layer, _TENSOR_IDS["down"], expert), (hidden, inner), WEIGHT_STD)


def router_bias(seed: int, layer: int, kind: str, experts=EXPERTS, alpha: float = ZIPF_ALPHA) -> np.ndarray | None:
    if kind == "none":
        return None
    rng = _rng(seed, layer, _TENSOR_IDS["bias"])
    if kind == "normal":
        return rng.standard_normal(experts, dtype=np.float32) * np.float32(0.5)
    if kind == "zipf":
        ranks = rng.permutation(experts) + 1
        p = ranks.astype(np.float64) ** -ZIPF_S
        p /= p.sum()
        return (alpha * np.log(p)).astype(np.float32)
    raise ValueError(f"unknown bias kind {kind!r}")


def hidden_states(seed: int, tokens: int, hidden=HIDDEN, step: int = 0) -> np.ndarray:
    return normal_bf16(seed, (step, _TENSOR_IDS["x"], tokens), (tokens, hidden), 1.0)


@dataclass
class LayerWeights:
    """Host copies of one layer (uint16 BF16 bits; bias FP32 or None)."""

    seed: int
    layer: int
    router: np.ndarray
    bias: np.ndarray | None
    sh_gate: np.ndarray
    sh_up: np.ndarray
    sh_down: np.ndarray
    sh_gate_w: np.ndarray
    gate_up: dict = field(default_factory=dict)
    down: dict = field(default_factory=dict)
    experts: int = EXPERTS
    hidden: int = HIDDEN
    inner: int = INNER

    def ensure(self, expert_ids) -> None:
        """Draw the named experts (lazily; cached)."""
        for e in sorted({int(e) for e in np.asarray(expert_ids).reshape(-1)}):
            if e not in self.gate_up:
                self.gate_up[e] = expert_gate_up(self.seed, self.layer, e, self.hidden, self.inner)
                self.down[e] = expert_down(self.seed, self.layer, e, self.hidden, self.inner)

    def stacked(self, threads: int = 0):
        """All experts as [E, 2I, H] and [E, H, I] uint16 arrays (drawn on a
        thread pool; each expert keeps its own seed, so the result does not
        depend on the thread count)."""
        import os
        from concurrent.futures import ThreadPoolExecutor

        gu = np.empty((self.experts, 2 * self.inner, self.hidden), dtype=np.uint16)
        dn = np.empty((self.experts, self.hidden, self.inner), dtype=np.uint16)

        def fill(e):
            gu[e] = self.gate_up[e] if e in self.gate_up else expert_gate_up(self.seed, self.layer, e, self.hidden,
                                                                              self.inner)
            dn[e] = self.down[e] if e in self.down else expert_down(self.seed, self.layer, e, self.hidden, self.inner)

        with ThreadPoolExecutor(threads or min(32, os.cpu_count() or 1)) as pool:
            list(pool.map(fill, range(self.experts)))
        return gu, dn


def layer_weights(seed: int, layer: int = 0, *, bias: str = "normal", experts=EXPERTS, hidden=HIDDEN,
                  inner=INNER, shared_inner=SHARED_INNER, alpha: float = ZIPF_ALPHA) -> LayerWeights:
    key = lambda name: (layer, _TENSOR_IDS[name])  # noqa: E731
    return LayerWeights(
        seed=seed, layer=layer,
        router=normal_bf16(seed, key("router"), (experts, hidden), WEIGHT_STD),
        bias=router_bias(seed, layer, bias, experts, alpha),
        sh_gate=normal_bf16(seed, key("sh_gate"), (shared_inner, hidden), WEIGHT_STD),
        sh_up=normal_bf16(seed, key("sh_up"), (shared_inner, hidden), WEIGHT_STD),
        sh_down=normal_bf16(seed, key("sh_down"), (hidden, shared_inner), WEIGHT_STD),
        sh_gate_w=normal_bf16(seed, key("sh_gate_w"), (hidden,), WEIGHT_STD),
        experts=experts, hidden=hidden, inner=inner,
    )


def calibrate_zipf_alpha(seed: int = 0, tokens: int = 4096, iters: int = 20) -> float:
    """Bisection on alpha so that the realised top-1 frequency of the most
    popular expert matches Zipf(1.1)'s first-rank share (reproduces ZIPF_ALPHA)."""
    w = layer_weights(seed, bias="none")
    x = bf16_bits_to_f32(hidden_states(seed, tokens))
    logits = bf16_bits_to_f32(f32_to_bf16_bits(x @ bf16_bits_to_f32(w.router).T))
    p = np.arange(1, EXPERTS + 1, dtype=np.float64) ** -ZIPF_S
    target = p[0] / p.sum()
    lo, hi = 0.0, 4.0
    for _ in range(iters):
        alpha = (lo + hi) / 2
        b = router_bias(seed, 0, "zipf", alpha=alpha)
        top1 = np.argmax(logits + b, axis=1)
        share = np.bincount(top1, minlength=EXPERTS).max() / tokens
        lo, hi = (alpha, hi) if share < target else (lo, alpha)
    return (lo + hi) / 2
