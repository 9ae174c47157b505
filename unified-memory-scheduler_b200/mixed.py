"""Mixed dense / MoE blocks with shared experts (DeepSeek-V2-Lite shape).

The reference's patched llama.cpp graph (build_moe_ffn plus the shared-expert branch,
third_party/patches/llama-b11669-hybrid-experts.patch:1394-1683 and the `ffn_*_shexp` tensors)
computes, for a MoE layer, moe_out = routed experts (softmax -> top-6, no renormalisation, x1.0)
and then moe_out + shared_out, where the shared experts are one SiLU FFN of width 2 x 1408; layer 0
is a plain dense FFN.  Both FFNs are one-expert, top-1 layers here: the softmax over one logit is
exactly 1.0 and the combine from 0.0f adds 1.0 * y, so they return the FFN's bits.
"""
from __future__ import annotations

import torch


class SharedExpertBlock:
    """out = routed(x) + shared(x), both MoeLayer handles on the same device (fp32 add, as ggml_add)."""

    def __init__(self, routed, shared):
        if shared.desc.experts != 1 or shared.desc.top_k != 1:
            raise ValueError("the shared-expert layer is a one-expert top-1 layer")
        if routed.desc.hidden != shared.desc.hidden:
            raise ValueError("routed and shared layers must share the model width")
        self.routed, self.shared = routed, shared

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        r = self.routed.forward(x, out=out, stream=stream)
        s = self.shared.forward(x, stream=stream)
        return r.add_(s)


class DenseFFN:
    """A dense SiLU FFN (layer 0 of the mixed model) run as a one-expert top-1 layer."""

    def __init__(self, layer):
        if layer.desc.experts != 1 or layer.desc.top_k != 1:
            raise ValueError("a dense FFN is a one-expert top-1 layer")
        self.layer = layer

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        return self.layer.forward(x, out=out, stream=stream)
