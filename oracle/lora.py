"""Multi-LoRA delta (oracle; test infrastructure only).

Restates src_ii/multi_lora.py MultiLoRALinear._compute_adapter_delta (:231-293)
and forward (:295-325) in torch on the CPU, keeping the reference's dtypes:
h = x @ A_j^T in bf16, contribution = (h @ B_j^T) * s_j (fp32 scale), rounded to
bf16 and summed in bf16, then added to the bf16 base output.
"""

from __future__ import annotations

import torch


def effective_scales(n_tokens, adapter_scales, token_to_image, lora_scalings, slot_active):
    scales = adapter_scales.unsqueeze(0) if adapter_scales.dim() == 1 else adapter_scales
    if token_to_image is not None:
        routing = token_to_image
        if n_tokens > routing.shape[0]:
            routing = routing.repeat(n_tokens // routing.shape[0])
    else:
        routing = torch.zeros(n_tokens, dtype=torch.long)
    valid = routing >= 0
    tok = scales[routing.clamp(min=0).long()] * valid.unsqueeze(1).to(scales.dtype)
    return tok * (lora_scalings * slot_active).unsqueeze(0)


def adapter_delta(x_2d, lora_A, lora_B, eff):
    """x_2d (n, in) bf16; lora_A list of (R, in); lora_B list of (out, R); eff (n, max_adapters)."""
    x_2d = x_2d.cpu()
    out = x_2d.new_zeros(x_2d.shape[0], lora_B[0].shape[0])
    for j in range(len(lora_A)):
        A, B = lora_A[j].cpu(), lora_B[j].cpu()
        h = (x_2d.float() @ A.float().t()).to(torch.bfloat16)
        contribution = (h.float() @ B.float().t()).to(torch.bfloat16).float() * eff[:, j].cpu().unsqueeze(1)
        out = out + contribution.to(out.dtype)
    return out
