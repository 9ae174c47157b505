"""Mixed dense / MoE stacks with shared experts: the DeepSeek-V2-Lite shape.

The reference's patched llama.cpp graph (build_moe_ffn plus the shared-expert branch,
third_party/patches/llama-b11669-hybrid-experts.patch:1394-1683, the `ffn_*_shexp` tensors of
tools/trace/make_moe_fixture.py:137-140) computes a MoE layer as moe_out = routed experts (softmax
-> top-6, no renormalisation, x1.0) and then moe_out + shared_out, where the two shared experts are
one SiLU FFN of width 2 x 1408; layer 0 is a plain dense FFN of width 10944.  Here every FFN is a
resident handle and the whole block is one umsx stack (umsx_stack_create_mixed): layer 0 and the
shared FFNs are one-expert top-1 layers (the softmax over one logit is exactly 1.0, so the combine
from 0.0f adds 1.0 * y = y), and each MoE layer's shared output is the term after the routed ones
in that layer's fused rank-order combine.
"""
from __future__ import annotations

from .configs import DEEPSEEK_V2_LITE, DEEPSEEK_V2_LITE_DENSE, DEEPSEEK_V2_LITE_SHARED
from .umsx import MoeLayer, MoeStack


def deepseek_v2_lite_layers(n_layers: int = 27, max_tokens: int = 1, device: int = 0, reserve_bytes: int = 1 << 30):
    """The configs[4] block as handles with seeded synthetic weights: (layers, shared) where layer 0
    is the dense FFN, layers 1.. the routed MoE layers, and shared[l] their shared FFNs (None at 0)."""
    layers, shared = [], []
    for l in range(n_layers):
        if l == 0:
            d = DEEPSEEK_V2_LITE_DENSE
            layers.append(MoeLayer(d.desc(max_tokens), synthetic=d.synthetic(layer=0), device=device,
                                   reserve_bytes=reserve_bytes))
            shared.append(None)
        else:
            r, s = DEEPSEEK_V2_LITE, DEEPSEEK_V2_LITE_SHARED
            layers.append(MoeLayer(r.desc(max_tokens), synthetic=r.synthetic(layer=l), device=device,
                                   reserve_bytes=reserve_bytes))
            shared.append(MoeLayer(s.desc(max_tokens), synthetic=s.synthetic(layer=l), device=device,
                                   reserve_bytes=reserve_bytes))
    return layers, shared


def deepseek_v2_lite_stack(n_layers: int = 27, max_tokens: int = 1, device: int = 0, rms_eps: float = 1e-5):
    """(stack, layers, shared): the configs[4] block as one stack (close the stack, then the handles)."""
    layers, shared = deepseek_v2_lite_layers(n_layers, max_tokens, device)
    return MoeStack(layers, max_tokens=max_tokens, rms_eps=rms_eps, shared=shared), layers, shared
