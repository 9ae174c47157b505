"""The benchmark layer shapes (seeded synthetic weights; no checkpoints are read).

Each entry gives the layer descriptor and the generator parameters used by
umsx_moe_create_synthetic.  Tensors are drawn by the counter-based generator
with stream = layer*16 + kind (kind 0 router W, 1 router bias, 2 gate_up or
gate, 3 up, 4 down, 5 gate/up bias, 6 down bias), so a host-side twin of the
generator reproduces any expert without generating the others.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .umsx import (ACT_SILU, ACT_SWIGLU_OAI, QUANT_MXFP4, QUANT_Q8_0, ROUTE_SOFTMAX_TOPK, ROUTE_SOFTMAX_TOPK_NORM,
                   ROUTE_TOPK_SOFTMAX, Desc)

KIND_ROUTER_W, KIND_ROUTER_B, KIND_GATE_UP, KIND_UP, KIND_DOWN, KIND_GU_BIAS, KIND_DOWN_BIAS = range(7)


def stream_id(layer: int, kind: int) -> int:
    return layer * 16 + kind


@dataclass
class LayerConfig:
    name: str
    hidden: int
    intermediate: int
    experts: int
    top_k: int
    quant: int
    routing: int
    activation: int
    fused_gate_up: bool
    has_bias: bool
    has_router_bias: bool
    seed: int
    layers: int = 1
    router_sigma: float = 0.02
    router_bias_sigma: float = 0.1
    bias_sigma: float = 0.02
    swiglu_alpha: float = 1.702
    swiglu_limit: float = 7.0
    routed_scale: float = 1.0
    tokens: tuple = field(default_factory=tuple)

    def desc(self, max_tokens: int, ep_rank: int = 0, ep_world: int = 1) -> Desc:
        return Desc(self.hidden, self.intermediate, self.experts, self.top_k, self.quant, self.routing,
                    self.activation, int(self.fused_gate_up), int(self.has_bias), int(self.has_router_bias),
                    self.swiglu_alpha, self.swiglu_limit, self.routed_scale, max_tokens, ep_rank, ep_world)

    def synthetic(self, layer: int = 0) -> dict:
        return dict(seed=self.seed, layer=layer, router_sigma=self.router_sigma,
                    router_bias_sigma=self.router_bias_sigma if self.has_router_bias else 0.0,
                    bias_sigma=self.bias_sigma)

    def expert_bytes(self) -> int:
        bb = 17 if self.quant == QUANT_MXFP4 else 34
        gu = 2 * self.intermediate * (self.hidden // 32) * bb
        dn = self.hidden * (self.intermediate // 32) * bb
        bias = (2 * self.intermediate + self.hidden) * 2 if self.has_bias else 0
        return gu + dn + bias

    def router_bytes(self) -> int:
        return self.experts * self.hidden * 4 + (self.experts * 4 if self.has_router_bias else 0)


# gpt-oss-20b-shaped layer, MXFP4, fused gate_up, SwiGLU-OAI, biases
GPT_OSS_20B = LayerConfig("gpt-oss-20b-layer", 2880, 2880, 32, 4, QUANT_MXFP4, ROUTE_TOPK_SOFTMAX, ACT_SWIGLU_OAI,
                          True, True, True, seed=0, tokens=(1, 32))
# Qwen3-30B-A3B-shaped layer, Q8_0, separate gate/up, SiLU, no biases
QWEN3_30B = LayerConfig("qwen3-30b-a3b-layer", 2048, 768, 128, 8, QUANT_Q8_0, ROUTE_SOFTMAX_TOPK_NORM, ACT_SILU,
                        False, False, False, seed=1, tokens=(1, 16, 512))
# GPT-OSS-120B-shaped 36-layer stack (weights as configs[0]), RMSNorm + residual
GPT_OSS_120B = LayerConfig("gpt-oss-120b-stack", 2880, 2880, 128, 4, QUANT_MXFP4, ROUTE_TOPK_SOFTMAX, ACT_SWIGLU_OAI,
                           True, True, True, seed=0, layers=36, tokens=(1, 64, 4096))
# load skew, Qwen3 shapes in Q8_0 and MXFP4; the router bias comes from zipf_router_bias
QWEN3_SKEW_Q8 = LayerConfig("qwen3-skew-q8_0", 2048, 768, 128, 8, QUANT_Q8_0, ROUTE_SOFTMAX_TOPK_NORM, ACT_SILU,
                            False, False, True, seed=3, tokens=(4096,))
QWEN3_SKEW_MXFP4 = LayerConfig("qwen3-skew-mxfp4", 2048, 768, 128, 8, QUANT_MXFP4, ROUTE_SOFTMAX_TOPK_NORM, ACT_SILU,
                               False, False, True, seed=3, tokens=(4096,))
# DeepSeek-V2-Lite-shaped routed layer, Q8_0, softmax -> top-6, no renorm, x1.0
DEEPSEEK_V2_LITE = LayerConfig("deepseek-v2-lite-layer", 2048, 1408, 64, 6, QUANT_Q8_0, ROUTE_SOFTMAX_TOPK, ACT_SILU,
                               False, False, False, seed=4, layers=27, tokens=(1, 2048))

CONFIGS = {c.name: c for c in (GPT_OSS_20B, QWEN3_30B, GPT_OSS_120B, QWEN3_SKEW_Q8, QWEN3_SKEW_MXFP4, DEEPSEEK_V2_LITE)}

# configs[4], the rest of the block: the two always-on shared experts (one FFN of width 2 x 1408,
# as the GGUF stores them) and the dense FFN of layer 0, each a one-expert top-1 layer (softmax
# over one logit is exactly 1.0, so its output is the FFN's)
DEEPSEEK_V2_LITE_SHARED = LayerConfig("deepseek-v2-lite-shared", 2048, 2 * 1408, 1, 1, QUANT_Q8_0, ROUTE_SOFTMAX_TOPK,
                                      ACT_SILU, False, False, False, seed=4, layers=27, tokens=(1, 2048))
DEEPSEEK_V2_LITE_DENSE = LayerConfig("deepseek-v2-lite-dense", 2048, 10944, 1, 1, QUANT_Q8_0, ROUTE_SOFTMAX_TOPK,
                                     ACT_SILU, False, False, False, seed=4, layers=1, tokens=(1, 2048))
CONFIGS.update({c.name: c for c in (DEEPSEEK_V2_LITE_SHARED, DEEPSEEK_V2_LITE_DENSE)})


def zipf_router_bias(experts: int, alpha: float = 1.2, noise_sigma: float = 0.5, seed: int = 3):
    """configs[3]'s router bias: log of a Zipf(alpha) expert popularity plus N(0, noise_sigma) noise,
    float32 [experts].  Popularity rank k (1 = hottest) has weight k^-alpha / sum_j j^-alpha; the
    ranks are a seeded random permutation of the experts, so the hot experts scatter over any
    contiguous expert-parallel partition.  With the router's own logits ~N(0, 0.02 * |x|) the top
    experts receive roughly 20x the mean load."""
    import numpy as np
    rng = np.random.default_rng(seed)
    ranks = rng.permutation(experts) + 1
    pop = ranks.astype(np.float64) ** -alpha
    pop /= pop.sum()
    return (np.log(pop) + rng.normal(0.0, noise_sigma, experts)).astype(np.float32)
