"""The reference's DiT block on the sm_100a kernels, with packed multi-image
sequences: drop-in for the block layer of src_ii/transformer.py.

* ``PackingInfo`` / ``pad_zimage`` / ``build_packed_sequence`` (:73-159): the
  packed layout [text_0, image_0, text_1, image_1, ...], each part padded to a
  multiple of ``pad_tokens_multiple`` with a pad token, document id = image index.
* ``JointAttention`` (:416-471): fused QKV FP8 linear -> P3 (per-head RMSNorm of
  Q/K + RoPE) -> block-masked quantized attention written in the (B, L, H * 128)
  row layout of the output linear -> output FP8 linear.
* ``FeedForward`` (:474-586): w1w3 FP8 GEMM with the SiLU-gate + 1 x 128 requant
  epilogue -> w2 FP8 GEMM (the reference's fused chain, one kernel shorter).
* ``JointTransformerBlock`` (:588-701): adaLN modulation, P1 norm-modulate (with
  the activation quantiser fused), attention, P2 gate + residual, FFN, P2.

adaLN parameters come in three forms, as in the reference:
  (B, dim)               per-batch: the fused per-sample kernels;
  (B, L, dim)            per-token tensors (the reference's pre-scattered form):
                         one row range per token;
  ``PerImageAdaLN``      the packed form this build uses: the (n_images, dim)
                         per-image rows plus the row ranges of the packed
                         sequence, applied without scattering them to
                         (L, dim) per layer (the reference scatters them,
                         src_ii/zimage_model.py:496-512).

Weights: the constructors mirror the reference (bf16 ``nn.Linear`` layers that a
reference state dict loads into); ``to_fp8()`` quantises them 128 x 128
(``quantize_fp8_blockwise``) and fuses w1/w3, after which every linear is an
``FP8Linear``.  ``replace_linear_with_fp8`` with an FP8 checkpoint works as well.
The forward needs FP8 linears (there is no bf16 GEMM path).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import _lib as L
from .fp8 import FP8Linear, quantize_fp8_blockwise_cuda
from .fp8_kernels import fp8_act_quant, fp8_gemm_blockwise, fp8_addmm_blockwise, fp8_gemm_silu_gate_quant
from .fused_kernels import (
    fused_qkv_postprocess,
    fused_rms_norm_gate_residual,
    fused_rms_norm_modulate,
    fused_rms_norm_modulate_quant,
    rms_norm_gate_residual_ranges,
    rms_norm_modulate_quant_ranges,
    rms_norm_modulate_ranges,
)
from .sage_attention import _attn_forward, _pv_for, attn_quant_out_from_streams, get_sage_config

HEAD_DIM = 128


# ---------------------------------------------------------------- packing
@dataclass
class PackingInfo:
    """How N (caption, image) pairs sit in one token sequence (reference :73-81)."""
    n_images: int
    segments: list[tuple[int, int, int, int]]  # (text_start, text_len, img_start, img_len)
    total_len: int
    document_id: Tensor                         # (total_len,) int32; -1 marks padding
    img_grid_sizes: list[tuple[int, int]]
    cap_lens: list[int]


def pad_zimage(feats: Tensor, pad_token: Tensor, pad_tokens_multiple: int) -> tuple[Tensor, int]:
    """Append copies of ``pad_token`` up to a multiple of ``pad_tokens_multiple``
    tokens (reference :93-98).  feats (B, n, dim) -> (B, n + pad, dim), pad."""
    pad = (-feats.shape[1]) % pad_tokens_multiple
    tail = pad_token.to(device=feats.device, dtype=feats.dtype).reshape(1, 1, -1).expand(feats.shape[0], pad, -1)
    return torch.cat((feats, tail), dim=1), pad


def build_packed_sequence(
    cap_feats_list: list[Tensor],
    img_patches_list: list[Tensor],
    img_grid_sizes: list[tuple[int, int]],
    cap_lens: list[int],
    pad_tokens_multiple: int,
    cap_pad_token: Tensor,
    x_pad_token: Tensor,
) -> tuple[Tensor, PackingInfo]:
    """Concatenate [caption_i, image_i] for every i, each padded (reference :117-159)."""
    parts: list[Tensor] = []
    segments: list[tuple[int, int, int, int]] = []
    doc: list[Tensor] = []
    pos = 0
    for i, (cap, img) in enumerate(zip(cap_feats_list, img_patches_list)):
        cap_p, _ = pad_zimage(cap, cap_pad_token, pad_tokens_multiple)
        img_p, _ = pad_zimage(img, x_pad_token, pad_tokens_multiple)
        nt, ni = cap_p.shape[1], img_p.shape[1]
        segments.append((pos, nt, pos + nt, ni))
        parts += [cap_p, img_p]
        doc.append(torch.full((nt + ni,), i, dtype=torch.int32))
        pos += nt + ni
    device = cap_feats_list[0].device
    info = PackingInfo(
        n_images=len(cap_feats_list), segments=segments, total_len=pos,
        document_id=torch.cat(doc).to(device), img_grid_sizes=list(img_grid_sizes), cap_lens=list(cap_lens),
    )
    return torch.cat(parts, dim=1), info


@dataclass
class RowRanges:
    """Row ranges of a packed sequence: rows [rows[i], rows[i + 1]) take
    parameter row param[i].  Both int32 on the device."""
    rows: Tensor
    param: Tensor
    n_params: int


def row_ranges(document_id: Tensor, n_params: int | None = None, device=None) -> RowRanges:
    """Runs of equal document id; padding tokens (id -1) take image 0's row, as the
    reference's per-token adaLN scatter remaps them (src_ii/zimage_model.py:496-500)."""
    d = document_id.detach().to("cpu", torch.int64).clone()
    d[d < 0] = 0
    n = d.numel()
    starts = torch.cat([torch.zeros(1, dtype=torch.int64), torch.nonzero(d[1:] != d[:-1]).flatten() + 1])
    rows = torch.cat([starts, torch.tensor([n])]).to(torch.int32)
    param = d[starts].to(torch.int32)
    dev = device if device is not None else document_id.device
    return RowRanges(rows.to(dev), param.to(dev), int(n_params if n_params is not None else int(d.max()) + 1))


@dataclass
class PerImageAdaLN:
    """One adaLN parameter of a packed sequence: per-image rows (n_images, dim)
    and the row ranges they apply to."""
    params: Tensor
    ranges: RowRanges


_IDENTITY_RANGES: dict[tuple[int, str], RowRanges] = {}


def _per_token_ranges(rows: int, device) -> RowRanges:
    key = (rows, str(device))
    r = _IDENTITY_RANGES.get(key)
    if r is None:
        ar = torch.arange(rows + 1, dtype=torch.int32, device=device)
        r = RowRanges(ar, ar[:-1].contiguous(), rows)
        _IDENTITY_RANGES[key] = r
    return r


def _as_ranges(p, x: Tensor) -> PerImageAdaLN | None:
    """PerImageAdaLN for a per-token parameter, None for a per-batch (B, dim) one."""
    if isinstance(p, PerImageAdaLN):
        return p
    if p.dim() == 3:
        dim = p.shape[-1]
        rows = x.numel() // dim
        assert p.numel() == rows * dim, f"per-token parameter {tuple(p.shape)} does not match x {tuple(x.shape)}"
        return PerImageAdaLN(p.reshape(rows, dim).contiguous(), _per_token_ranges(rows, x.device))
    return None


def modulate_quant(x: Tensor, weight: Tensor, scale, eps: float) -> tuple[Tensor, Tensor]:
    """rmsnorm(x) * w * (1 + scale) -> 1 x 128 e4m3 codes and scales."""
    r = _as_ranges(scale, x)
    if r is None:
        return fused_rms_norm_modulate_quant(x, weight, scale.contiguous(), eps)
    return rms_norm_modulate_quant_ranges(x, weight, r.params, r.ranges.rows, r.ranges.param, eps)


def modulate(x: Tensor, weight: Tensor, scale, eps: float) -> Tensor:
    r = _as_ranges(scale, x)
    if r is None:
        return fused_rms_norm_modulate(x, weight, scale.contiguous(), eps)
    return rms_norm_modulate_ranges(x, weight, r.params, r.ranges.rows, r.ranges.param, eps)


def gate_residual(x: Tensor, weight: Tensor, gate, residual: Tensor, eps: float) -> Tensor:
    """residual + tanh(gate) * rmsnorm(x) * w."""
    r = _as_ranges(gate, x)
    if r is None:
        return fused_rms_norm_gate_residual(x, weight, gate.contiguous(), residual, eps)
    return rms_norm_gate_residual_ranges(x, weight, r.params, residual, r.ranges.rows, r.ranges.param, eps)


# ---------------------------------------------------------------- modules
class RMSNormModule(nn.Module):
    """rmsnorm(x) * w (reference :305-317), on the P1 kernel with scale 0
    (1 + 0 is exact)."""

    def __init__(self, dim: int, eps: float = 1e-5, elementwise_affine: bool = True, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(dim, device=device, dtype=dtype))
        else:
            self.register_buffer("weight", torch.ones(dim, device=device, dtype=dtype))

    def forward(self, x: Tensor) -> Tensor:
        shp = x.shape
        x3 = x.reshape(-1, 1, shp[-1]).contiguous() if x.dim() != 3 else x.contiguous()
        zero = torch.zeros(x3.shape[0], shp[-1], dtype=torch.float32, device=x.device)
        return fused_rms_norm_modulate(x3, self.weight, zero, self.eps).reshape(shp)


def _fp8(lin: nn.Module) -> FP8Linear:
    if isinstance(lin, FP8Linear):
        return lin
    if isinstance(lin, nn.Linear):
        w8, ws = quantize_fp8_blockwise_cuda(lin.weight.detach())
        bias = None if lin.bias is None else lin.bias.detach().to(torch.bfloat16)
        return FP8Linear(w8, ws, bias)
    return lin  # e.g. MultiLoRALinear: called as a module


def _linear_codes(a8: Tensor, a_s: Tensor, lin: FP8Linear) -> Tensor:
    if lin.bias is not None:
        return fp8_addmm_blockwise(a8, a_s, lin.weight, lin.weight_scale, bias=lin.bias,
                                   output_dtype=lin.output_dtype)
    return fp8_gemm_blockwise(a8, a_s, lin.weight, lin.weight_scale, output_dtype=lin.output_dtype)


def _is_plain_fp8(lin) -> bool:
    return isinstance(lin, FP8Linear) and not getattr(lin, "_transposed", False)


class JointAttention(nn.Module):
    """Fused-QKV, block-masked attention (reference :416-471)."""

    def __init__(self, dim: int, n_heads: int, n_kv_heads: int | None, qk_norm: bool,
                 out_bias: bool = False, use_sage: bool = True, device=None, dtype=None):
        super().__init__()
        self.n_kv_heads = n_heads if n_kv_heads is None else n_kv_heads
        if self.n_kv_heads != n_heads:
            raise ValueError("JointAttention: grouped K/V heads are not supported (fused QKV is 3 * dim)")
        self.n_local_heads = n_heads
        self.n_local_kv_heads = self.n_kv_heads
        self.n_rep = 1
        self.head_dim = dim // n_heads
        if self.head_dim != HEAD_DIM:
            raise ValueError(f"head_dim must be {HEAD_DIM}, got {self.head_dim}")
        if not use_sage:
            raise ValueError("JointAttention: only the quantized (sage) attention backend is built")
        self.use_sage = True
        if not qk_norm:
            # the fused P3 kernel always normalises Q and K; the reference's
            # nn.Identity q/k norm has no fused counterpart there either
            raise ValueError("JointAttention: qk_norm=False is not supported by the fused QKV post-process")
        self.qkv = nn.Linear(dim, 3 * dim, bias=False, device=device, dtype=dtype)
        self.out = nn.Linear(dim, dim, bias=out_bias, device=device, dtype=dtype)
        self.q_norm = RMSNormModule(self.head_dim, elementwise_affine=True, device=device, dtype=dtype)
        self.k_norm = RMSNormModule(self.head_dim, elementwise_affine=True, device=device, dtype=dtype)

    def to_fp8(self) -> "JointAttention":
        self.qkv = _fp8(self.qkv)
        self.out = _fp8(self.out)
        return self

    def _qkv(self, qkv: Tensor, freqs_cis: Tensor):
        return fused_qkv_postprocess(qkv, self.q_norm.weight, self.k_norm.weight, freqs_cis,
                                     self.n_local_heads, self.head_dim, self.q_norm.eps)

    def core(self, qkv: Tensor, freqs_cis: Tensor, block_mask: Tensor) -> Tensor:
        """(B, L, 3 dim) bf16 -> attention output (B, L, dim) bf16 in the row layout
        of the output linear (the reference's transpose + reshape, :466)."""
        xq, xk, xv = self._qkv(qkv, freqs_cis)
        # sage_attn_masked_op: INT8 QK, bf16 PV (or the per-block variant)
        cfg = get_sage_config()
        o, _ = _attn_forward(xq, xk, xv, 1.0 / (self.head_dim ** 0.5), block_mask=block_mask, qk_quant="int8",
                             pv_quant=_pv_for("bf16"), granularity=cfg["qk_granularity"], want_lse=False,
                             out_bnhd=True)
        return o

    def core_codes(self, qkv: Tensor, freqs_cis: Tensor, block_mask: Tensor) -> tuple[Tensor, Tensor]:
        """``core`` with the output written as the output linear's 1 x 128 e4m3 input
        (codes (B, L, dim), scales (B, L, dim / 128)), equal to fp8_act_quant(core(...))."""
        B, Lq, dim = qkv.shape[0], qkv.shape[1], qkv.shape[2] // 3
        o8 = torch.empty(B, Lq, dim, dtype=torch.float8_e4m3fn, device=qkv.device)
        o_s = torch.empty(B, Lq, dim // 128, dtype=torch.float32, device=qkv.device)
        cfg = get_sage_config()
        # P3 fused with the quantisation prologue, then the quantised-output attention
        attn_quant_out_from_streams([(qkv.contiguous(), self.q_norm.weight, self.k_norm.weight, freqs_cis, 0,
                                      self.q_norm.eps)], self.n_local_heads, Lq, 1.0 / (self.head_dim ** 0.5),
                                    block_mask=block_mask, qk_quant="int8", pv_quant=_pv_for("bf16"),
                                    granularity=cfg["qk_granularity"], regions=[(o8, o_s)])
        return o8, o_s

    def forward(self, x: Tensor, x_mask: Tensor | None, freqs_cis: Tensor, block_mask=None,
                adapter_scales: Tensor | None = None, token_to_image: Tensor | None = None) -> Tensor:
        if block_mask is None:
            raise RuntimeError("JointAttention requires a block mask")
        if adapter_scales is not None:
            qkv = self.qkv(x, adapter_scales=adapter_scales, token_to_image=token_to_image)
        else:
            qkv = self.qkv(x)
        o = self.core(qkv, freqs_cis, block_mask)
        if adapter_scales is not None:
            return self.out(o, adapter_scales=adapter_scales, token_to_image=token_to_image)
        return self.out(o)

    def forward_codes(self, a8: Tensor, a_s: Tensor, freqs_cis: Tensor, block_mask: Tensor) -> Tensor:
        """Attention on an input already quantised 1 x 128 (the fused norm's output)."""
        if block_mask is None:
            raise RuntimeError("JointAttention requires a block mask")
        qkv = _linear_codes(a8, a_s, self.qkv)
        if _is_plain_fp8(self.out):
            return _linear_codes(*self.core_codes(qkv, freqs_cis, block_mask), self.out)
        return self.out(self.core(qkv, freqs_cis, block_mask))


class FeedForward(nn.Module):
    """SiLU-gated FFN (reference :474-586): w2(silu(w1 x) * w3 x)."""

    def __init__(self, dim: int, hidden_dim: int, multiple_of: int, ffn_dim_multiplier: float | None,
                 device=None, dtype=None):
        super().__init__()
        if ffn_dim_multiplier is not None:
            hidden_dim = int(ffn_dim_multiplier * hidden_dim)
        hidden_dim = multiple_of * ((hidden_dim + multiple_of - 1) // multiple_of)
        self.w1 = nn.Linear(dim, hidden_dim, bias=False, device=device, dtype=dtype)
        self.w2 = nn.Linear(hidden_dim, dim, bias=False, device=device, dtype=dtype)
        self.w3 = nn.Linear(dim, hidden_dim, bias=False, device=device, dtype=dtype)
        self.hidden_dim = hidden_dim
        self._fused = False
        self._fused_chain = False

    def fuse_w1w3(self) -> None:
        """w1 and w3 as one (2 hidden, dim) FP8 linear (reference :495-524)."""
        if self._fused:
            return
        w1, w3 = _fp8(self.w1), _fp8(self.w3)
        self.w1w3 = FP8Linear(torch.cat([w1.weight, w3.weight], 0), torch.cat([w1.weight_scale, w3.weight_scale], 0),
                              bias=None, block_size=w1.block_size, output_dtype=w1.output_dtype)
        del self.w1
        del self.w3
        self._fused = True

    def enable_fused_chain(self) -> None:
        if self._fused and isinstance(self.w2, FP8Linear):
            self._fused_chain = True

    def to_fp8(self) -> "FeedForward":
        self.fuse_w1w3()
        self.w2 = _fp8(self.w2)
        self.enable_fused_chain()
        return self

    def forward_codes(self, a8: Tensor, a_s: Tensor) -> Tensor:
        """FFN on a quantised input: w1w3 GEMM + SiLU gate + requant in one kernel, then w2."""
        g8, g_s = fp8_gemm_silu_gate_quant(a8, a_s, self.w1w3.weight, self.w1w3.weight_scale)
        return _linear_codes(g8, g_s, self.w2)

    def forward(self, x: Tensor, adapter_scales: Tensor | None = None,
                token_to_image: Tensor | None = None) -> Tensor:
        if not self._fused_chain:
            raise RuntimeError("FeedForward: call to_fp8() (FP8 weights, fused w1w3 chain) first")
        if adapter_scales is not None:
            raise NotImplementedError("FeedForward: adapter scales need MultiLoRALinear layers")
        a8, a_s = fp8_act_quant(x.contiguous())
        return self.forward_codes(a8, a_s)


class JointTransformerBlock(nn.Module):
    """The reference's DiT block (src_ii/transformer.py:588-701)."""

    def __init__(self, layer_id: int, dim: int, n_heads: int, n_kv_heads: int | None, multiple_of: int,
                 ffn_dim_multiplier: float | None, norm_eps: float, qk_norm: bool, modulation: bool = True,
                 z_image_modulation: bool = False, attn_out_bias: bool = False, use_sage: bool = True,
                 device=None, dtype=None):
        super().__init__()
        self.dim = dim
        self.head_dim = dim // n_heads
        self.attention = JointAttention(dim, n_heads, n_kv_heads, qk_norm, out_bias=attn_out_bias,
                                        use_sage=use_sage, device=device, dtype=dtype)
        self.feed_forward = FeedForward(dim, dim, multiple_of, ffn_dim_multiplier, device=device, dtype=dtype)
        self.layer_id = layer_id
        self.attention_norm1 = RMSNormModule(dim, eps=norm_eps, device=device, dtype=dtype)
        self.ffn_norm1 = RMSNormModule(dim, eps=norm_eps, device=device, dtype=dtype)
        self.attention_norm2 = RMSNormModule(dim, eps=norm_eps, device=device, dtype=dtype)
        self.ffn_norm2 = RMSNormModule(dim, eps=norm_eps, device=device, dtype=dtype)
        self.modulation = modulation
        self.z_image_modulation = z_image_modulation
        if modulation:
            if z_image_modulation:
                self.adaLN_modulation = nn.Sequential(
                    nn.Linear(min(dim, 256), 4 * dim, bias=True, device=device, dtype=dtype))
            else:
                self.adaLN_modulation = nn.Sequential(
                    nn.SiLU(), nn.Linear(min(dim, 1024), 4 * dim, bias=True, device=device, dtype=dtype))

    def to_fp8(self) -> "JointTransformerBlock":
        self.attention.to_fp8()
        self.feed_forward.to_fp8()
        return self

    def adaln_params(self, adaln_input: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        """(n, 256 or 1024) -> scale_msa, gate_msa, scale_mlp, gate_mlp, each (n, dim)
        contiguous (one cuBLAS bf16 GEMM: the P4 adaLN projection)."""
        return tuple(t.contiguous() for t in self.adaLN_modulation(adaln_input).chunk(4, dim=1))

    def forward(self, x: Tensor, x_mask: Tensor | None, freqs_cis: Tensor, adaln_input: Tensor | None = None,
                precomputed_adaln=None, block_mask=None, adapter_scales: Tensor | None = None,
                token_to_image: Tensor | None = None) -> Tensor:
        eps1, eps2 = self.attention_norm1.eps, self.attention_norm2.eps
        if not self.modulation:
            # context refiner: x + n2(attn(n1(x))), x + n2'(ffn(n1'(x)))
            assert adaln_input is None
            a = self.attention(self.attention_norm1(x), x_mask, freqs_cis, block_mask=block_mask,
                               adapter_scales=adapter_scales, token_to_image=token_to_image)
            x = x + self.attention_norm2(a)
            f = self.feed_forward(self.ffn_norm1(x), adapter_scales=adapter_scales, token_to_image=token_to_image)
            return x + self.ffn_norm2(f)
        if precomputed_adaln is not None:
            scale_msa, gate_msa, scale_mlp, gate_mlp = precomputed_adaln
        else:
            assert adaln_input is not None
            scale_msa, gate_msa, scale_mlp, gate_mlp = self.adaln_params(adaln_input)
        x = x.contiguous()
        att, ffn = self.attention, self.feed_forward
        if adapter_scales is None and _is_plain_fp8(att.qkv) and ffn._fused_chain and _is_plain_fp8(ffn.w1w3):
            # every linear is FP8: the norms emit the quantised GEMM inputs directly
            a8, a_s = modulate_quant(x, self.attention_norm1.weight, scale_msa, eps1)
            attn_out = att.forward_codes(a8, a_s, freqs_cis, block_mask)
            x = gate_residual(attn_out, self.attention_norm2.weight, gate_msa, x, eps2)
            f8, f_s = modulate_quant(x, self.ffn_norm1.weight, scale_mlp, self.ffn_norm1.eps)
            ffn_out = ffn.forward_codes(f8, f_s)
            return gate_residual(ffn_out, self.ffn_norm2.weight, gate_mlp, x, self.ffn_norm2.eps)
        attn_in = modulate(x, self.attention_norm1.weight, scale_msa, eps1)
        attn_out = att(attn_in, x_mask, freqs_cis, block_mask=block_mask, adapter_scales=adapter_scales,
                       token_to_image=token_to_image)
        x = gate_residual(attn_out, self.attention_norm2.weight, gate_msa, x, eps2)
        ffn_in = modulate(x, self.ffn_norm1.weight, scale_mlp, self.ffn_norm1.eps)
        ffn_out = ffn(ffn_in, adapter_scales=adapter_scales, token_to_image=token_to_image)
        return gate_residual(ffn_out, self.ffn_norm2.weight, gate_mlp, x, self.ffn_norm2.eps)


def per_image_adaln(block: JointTransformerBlock, adaln_inputs: Tensor, ranges: RowRanges
                    ) -> tuple[PerImageAdaLN, PerImageAdaLN, PerImageAdaLN, PerImageAdaLN]:
    """The block's four adaLN parameters for a packed sequence: one row per image
    (adaln_inputs (n_images, 256)), applied to the image's row ranges."""
    return tuple(PerImageAdaLN(p, ranges) for p in block.adaln_params(adaln_inputs))


def build_packed_rope(packing_info: PackingInfo, axes_dim=(32, 48, 48), theta: float = 256.0, device=None) -> Tensor:
    """RoPE rotations of a packed sequence, (1, total_len, 1, 64, 2, 2) fp32
    (reference build_packed_rope, src_ii/transformer.py:162-197, with EmbedND
    :331-344): caption token t has position (t + 1, 0, 0); image token (r, c) has
    (padded caption length + 1, r, c); padding tokens have position 0."""
    from .attention import rope_embed

    dev = device if device is not None else packing_info.document_id.device
    pos = torch.zeros(packing_info.total_len, 3, dtype=torch.float32, device=dev)
    for i, (ts, tl, is_, _il) in enumerate(packing_info.segments):
        H_t, W_t = packing_info.img_grid_sizes[i]
        pos[ts:ts + tl, 0] = torch.arange(tl, dtype=torch.float32, device=dev) + 1.0
        n = H_t * W_t
        pos[is_:is_ + n, 0] = tl + 1
        pos[is_:is_ + n, 1] = torch.arange(H_t, dtype=torch.float32, device=dev).repeat_interleave(W_t)
        pos[is_:is_ + n, 2] = torch.arange(W_t, dtype=torch.float32, device=dev).repeat(H_t)
    f = torch.cat([rope_embed(pos[:, a], d, theta) for a, d in enumerate(axes_dim)], dim=-3)
    return f.reshape(1, packing_info.total_len, 1, sum(axes_dim) // 2, 2, 2).contiguous()


class PackedTrunk(nn.Module):
    """``n_layers`` JointTransformerBlocks over one packed sequence: the main layer
    loop of the reference model (src_ii/zimage_model.py:680-702) with its
    per-token adaLN for packed multi-image inputs (:480-512) and the batched adaLN
    projection of all layers in one GEMM (:194-248).

    forward(x (1, L, dim) bf16, adaln_inputs (n_images, 256), ranges, block_mask,
    freqs (1, L, 1, 64, 2, 2)): with ``ranges`` (row_ranges of the plan's
    document ids) every image gets its own modulation; with ranges None the
    adaLN inputs are per batch row (B, 256) for a (B, L, dim) input."""

    def __init__(self, n_layers: int, dim: int, n_heads: int, multiple_of: int = 256,
                 ffn_dim_multiplier: float | None = 8.0 / 3.0, norm_eps: float = 1e-5, seed: int = 0,
                 device=None):
        super().__init__()
        dev = torch.device(device) if device is not None else torch.device("cpu")
        # seeded random init without disturbing the caller's RNG streams
        with torch.random.fork_rng(devices=[dev] if dev.type == "cuda" else []):
            torch.manual_seed(seed)
            self.layers = nn.ModuleList([
                JointTransformerBlock(i, dim, n_heads, None, multiple_of, ffn_dim_multiplier, norm_eps,
                                      qk_norm=True, modulation=True, z_image_modulation=True, device=device,
                                      dtype=torch.bfloat16).to_fp8()
                for i in range(n_layers)])
        self.dim = dim
        self._adaln_w: Tensor | None = None
        self._adaln_b: Tensor | None = None

    def _adaln_all(self, adaln_inputs: Tensor) -> list[tuple[Tensor, Tensor, Tensor, Tensor]]:
        if self._adaln_w is None:
            lins = [blk.adaLN_modulation[-1] for blk in self.layers]
            self._adaln_w = torch.cat([l.weight.detach() for l in lins], 0).contiguous()
            self._adaln_b = torch.cat([l.bias.detach() for l in lins], 0).contiguous()
        mod = F.linear(adaln_inputs.to(self._adaln_w.dtype), self._adaln_w, self._adaln_b)
        D = self.dim
        return [tuple(mod[:, (4 * j + c) * D:(4 * j + c + 1) * D].contiguous() for c in range(4))
                for j in range(len(self.layers))]

    def forward(self, x: Tensor, adaln_inputs: Tensor, ranges: RowRanges | None, block_mask: Tensor,
                freqs: Tensor) -> Tensor:
        params = self._adaln_all(adaln_inputs)
        for blk, p in zip(self.layers, params):
            pre = tuple(PerImageAdaLN(t, ranges) for t in p) if ranges is not None else p
            x = blk(x, None, freqs, precomputed_adaln=pre, block_mask=block_mask)
        return x
