"""Diffusion-transformer workloads on the futudiffu_b200 kernels.

The benchmark models of the quantized DiT hot path, built from random-init
weights (no checkpoint is needed or read):

* ``DoubleStreamBlock`` -- the MMDiT double-stream block: text and image
  streams with their own weights, joint quantized attention over both.
* ``SingleStreamBlock`` -- the single-stream block: one fused QKV + MLP-in
  linear, attention and GELU(tanh) MLP in parallel, one fused output linear.
* ``DiT`` + ``euler_denoise`` -- the 12B-class rectified-flow transformer
  (19 double + 38 single blocks at hidden 3072) and its Euler sampler.

Block anatomy follows the reference's Z-Image transformer
(src_ii/transformer.py:459-475, :533-567, :680-702): adaLN from a timestep
vector produces per-sublayer (scale, gate) pairs consumed by
``fused_rms_norm_modulate`` (x -> rmsnorm(x) w (1 + scale)) and
``fused_rms_norm_gate_residual`` (r + tanh(gate) rmsnorm(y) w); Q/K get a
per-head RMSNorm and RoPE inside ``fused_qkv_postprocess``; every linear of the
blocks is an FP8 128 x 128 block-scaled GEMM.  The FFN chain stays in FP8
between its two GEMMs: the first GEMM's epilogue applies GELU(tanh) and the
1 x 128 requantisation (``fp8_gemm_gelu_tanh_quant``), the second consumes the
codes directly.  Small per-sample GEMMs (timestep MLP, adaLN, patch in/out
projections) run in bf16 through torch; they are not on the hot path.

Every hot op is one of the package's sm_100a kernels; nothing here has a CPU
path (the CPU restatement used for checking lives with the test oracle).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from . import _lib as L
from .attention import rope_embed
from .fp8 import FP8Linear, quantize_fp8_blockwise_cuda
from .fp8_kernels import (
    fp8_act_quant,
    fp8_addmm_blockwise,
    fp8_gemm_blockwise,
    fp8_gemm_gelu_tanh_quant,
    fp8_gemm_grouped2,
)
from .fused_kernels import (
    fused_qkv_postprocess,
    fused_rms_norm_gate_residual,
    fused_rms_norm_modulate,
    fused_rms_norm_modulate_quant,
    qkv_postprocess_into,
)
from .sage_attention import (
    _attn_forward,
    attn_forward_quant_out,
    attn_quant_out_from_linear,
    attn_quant_out_from_streams,
    fused_prologue_ok,
    linear_prologue_ok,
)

HEAD_DIM = 128


@dataclass
class DiTConfig:
    hidden: int = 3072
    heads: int = 24
    mlp_ratio: int = 4
    n_double: int = 19
    n_single: int = 38
    txt_tokens: int = 512
    img_grid: tuple[int, int] = (64, 64)  # token grid after 2x2 patching
    patch_dim: int = 64                    # 16 latent channels x 2 x 2
    time_dim: int = 256
    rope_axes: tuple[int, int] = (64, 64)  # head_dim split over the (h, w) axes
    rope_theta: float = 10000.0
    eps: float = 1e-5
    # quantized attention mode: INT8 per-block Q/K codes, bf16 P and V (within
    # cosine 0.9995 of the oracle at the benchmark shapes; pv_quant="fp8" selects
    # e4m3 P/V, about 2 % faster in the attention kernel, whose rounding noise is
    # larger than that tolerance)
    qk_quant: str = "int8"
    pv_quant: str = "bf16"
    granularity: str = "per_block"

    @property
    def img_tokens(self) -> int:
        return self.img_grid[0] * self.img_grid[1]

    @property
    def tokens(self) -> int:
        return self.txt_tokens + self.img_tokens


def random_fp8_linear(out_f: int, in_f: int, gen: torch.Generator, device, std: float = 0.02,
                      bias: bool = False) -> FP8Linear:
    """An FP8Linear whose weight is N(0, std) quantised 128 x 128 on the device."""
    w = torch.randn(out_f, in_f, generator=gen, device=device, dtype=torch.float32).mul_(std)
    w8, ws = quantize_fp8_blockwise_cuda(w.to(torch.bfloat16))
    b = None
    if bias:
        b = (torch.randn(out_f, generator=gen, device=device) * std).to(torch.bfloat16)
    return FP8Linear(w8, ws, b)


def _rand(shape, gen, device, std, mean=0.0, dtype=torch.bfloat16) -> Tensor:
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std + mean).to(dtype)


def f32_norms(m: nn.Module) -> tuple[Tensor, Tensor]:
    """f32 copies of a block's Q/K norm weights for the P3 kernels (which read f32;
    handing them the bf16 parameters costs two conversion launches per attention).
    Made on first use and remade only when a parameter changes: the cache key is
    each parameter's storage address and version counter, so a weight load (in
    place or by assignment) or a move to another device is picked up."""
    qn, kn = m.q_norm, m.k_norm
    key = (qn.data_ptr(), qn._version, kn.data_ptr(), kn._version)
    cache = m.__dict__.get("_norm32")
    if cache is None or cache[0] != key:
        cache = (key, qn.detach().float(), kn.detach().float())
        m.__dict__["_norm32"] = cache
    return cache[1], cache[2]


def image_freqs(cfg: DiTConfig, device) -> Tensor:
    """2-D RoPE rotations of the image tokens, (img_tokens, head_dim/2, 2, 2) fp32."""
    gh, gw = cfg.img_grid
    ys = torch.arange(gh, device=device).repeat_interleave(gw)
    xs = torch.arange(gw, device=device).repeat(gh)
    fy = rope_embed(ys, cfg.rope_axes[0], cfg.rope_theta)
    fx = rope_embed(xs, cfg.rope_axes[1], cfg.rope_theta)
    return torch.cat([fy, fx], dim=-3).contiguous()


def batch_freqs(freqs: Tensor, B: int) -> Tensor:
    """Per-sequence rotations (L, 64, 2, 2) repeated for a batch: (B, L, 64, 2, 2) contiguous."""
    return freqs.unsqueeze(0).expand(B, *freqs.shape).contiguous()


def text_freqs(cfg: DiTConfig, device) -> Tensor:
    """Text tokens carry no positional rotation: identity matrices."""
    eye = torch.eye(2, dtype=torch.float32, device=device)
    return eye.expand(cfg.txt_tokens, HEAD_DIM // 2, 2, 2).contiguous()


def linear_bf16(x: Tensor, lin: FP8Linear) -> Tensor:
    """x (..., K) bf16 -> FP8 GEMM -> (..., N) bf16 (activation quantised 1 x 128)."""
    a8, a_s = fp8_act_quant(x)
    if lin.bias is not None:
        return fp8_addmm_blockwise(a8, a_s, lin.weight, lin.weight_scale, bias=lin.bias,
                                   output_dtype=torch.bfloat16)
    return fp8_gemm_blockwise(a8, a_s, lin.weight, lin.weight_scale, output_dtype=torch.bfloat16)


def gemm_bf16(a8: Tensor, a_s: Tensor, lin: FP8Linear) -> Tensor:
    """Quantised activation (codes, 1 x 128 scales) -> FP8 GEMM -> bf16."""
    if lin.bias is not None:
        return fp8_addmm_blockwise(a8, a_s, lin.weight, lin.weight_scale, bias=lin.bias,
                                   output_dtype=torch.bfloat16)
    return fp8_gemm_blockwise(a8, a_s, lin.weight, lin.weight_scale, output_dtype=torch.bfloat16)


def mlp_fp8_q(a8: Tensor, a_s: Tensor, w_in: FP8Linear, w_out: FP8Linear) -> Tensor:
    """GELU(tanh) MLP on a quantised input, kept in FP8 between its GEMMs."""
    h8, h_s = fp8_gemm_gelu_tanh_quant(a8, a_s, w_in.weight, w_in.weight_scale, bias=w_in.bias)
    return fp8_gemm_blockwise(h8, h_s, w_out.weight, w_out.weight_scale, output_dtype=torch.bfloat16)


def mlp_fp8(x: Tensor, w_in: FP8Linear, w_out: FP8Linear) -> Tensor:
    """GELU(tanh) MLP kept in FP8 between its GEMMs (fused GELU + requant epilogue)."""
    a8, a_s = fp8_act_quant(x)
    h8, h_s = fp8_gemm_gelu_tanh_quant(a8, a_s, w_in.weight, w_in.weight_scale, bias=w_in.bias)
    return fp8_gemm_blockwise(h8, h_s, w_out.weight, w_out.weight_scale, output_dtype=torch.bfloat16)


def joint_attention(q: Tensor, k: Tensor, v: Tensor, cfg: DiTConfig) -> Tensor:
    """Quantized attention over (B, H, N, 128) -> (B, N, H * 128) bf16, written in
    that layout by the kernel (no transpose)."""
    o, _ = _attn_forward(q, k, v, None, block_mask=None, qk_quant=cfg.qk_quant, pv_quant=cfg.pv_quant,
                         granularity=cfg.granularity, want_lse=False, out_bnhd=True)
    return o


def joint_prologue_attention(streams, cfg: DiTConfig, N: int, regions, split=None) -> None:
    """Attention straight from the QKV linear outputs of the streams of a joint
    attention: P3 fused with the quantisation prologue when the streams are
    128-row aligned (else P3 into joint Q/K/V buffers and the separate prologue),
    output written as the out-projections' 1 x 128 e4m3 input into ``regions``."""
    if fused_prologue_ok([st[0].shape[1] for st in streams]):
        attn_quant_out_from_streams(streams, cfg.heads, N, None, block_mask=None, qk_quant=cfg.qk_quant,
                                    pv_quant=cfg.pv_quant, granularity=cfg.granularity, regions=regions,
                                    split=split)
        return
    B, dev = streams[0][0].shape[0], streams[0][0].device
    q, k, v = (torch.empty(B, cfg.heads, N, HEAD_DIM, dtype=torch.bfloat16, device=dev) for _ in range(3))
    for qkv, qn, kn, fr, off, eps in streams:
        qkv_postprocess_into(qkv, qn, kn, fr, q, k, v, off, eps)
    joint_attention_codes(q, k, v, cfg, regions, split)


def joint_attention_codes(q: Tensor, k: Tensor, v: Tensor, cfg: DiTConfig, regions, split=None) -> None:
    """Quantized attention written straight as the output linears' 1 x 128 e4m3
    input (codes + scales) into ``regions`` (see attn_forward_quant_out)."""
    attn_forward_quant_out(q, k, v, None, block_mask=None, qk_quant=cfg.qk_quant, pv_quant=cfg.pv_quant,
                           granularity=cfg.granularity, regions=regions, split=split)


class _Stream(nn.Module):
    """Weights of one stream of a double-stream block."""

    def __init__(self, cfg: DiTConfig, gen, device):
        super().__init__()
        D = cfg.hidden
        self.adaln = nn.Linear(D, 4 * D, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            self.adaln.weight.copy_(_rand((4 * D, D), gen, device, 0.02))
            self.adaln.bias.copy_(_rand((4 * D,), gen, device, 0.02))
        self.norm_w = nn.ParameterList(
            [nn.Parameter(_rand((D,), gen, device, 0.05, 1.0), requires_grad=False) for _ in range(4)])
        self.q_norm = nn.Parameter(_rand((HEAD_DIM,), gen, device, 0.05, 1.0), requires_grad=False)
        self.k_norm = nn.Parameter(_rand((HEAD_DIM,), gen, device, 0.05, 1.0), requires_grad=False)
        self.qkv = random_fp8_linear(3 * D, D, gen, device)
        self.proj = random_fp8_linear(D, D, gen, device)
        self.mlp_in = random_fp8_linear(cfg.mlp_ratio * D, D, gen, device)
        self.mlp_out = random_fp8_linear(D, cfg.mlp_ratio * D, gen, device)

    def modulation(self, vec: Tensor) -> list[Tensor]:
        # (scale_attn, gate_attn, scale_mlp, gate_mlp), each (B, D)
        return list(self.adaln(torch.nn.functional.silu(vec)).chunk(4, dim=-1))


class DoubleStreamBlock(nn.Module):
    """MMDiT double-stream block: per-stream weights, joint attention."""

    def __init__(self, cfg: DiTConfig, gen, device):
        super().__init__()
        self.cfg = cfg
        self.txt = _Stream(cfg, gen, device)
        self.img = _Stream(cfg, gen, device)

    def forward(self, x_txt: Tensor, x_img: Tensor, vec: Tensor, freqs_txt: Tensor,
                freqs_img: Tensor, mods: Tensor | None = None) -> tuple[Tensor, Tensor]:
        """x_* (B, L_*, D) bf16; vec (B, D); freqs_* (B, L_*, 64, 2, 2) fp32 (see batch_freqs);
        mods: this block's modulation precomputed as (8, B, D) (text stream's four
        chunks, then the image stream's; see DiT.modulations), else computed from vec."""
        cfg = self.cfg
        B, Nt = x_txt.shape[0], x_txt.shape[1]
        N = Nt + x_img.shape[1]
        sts, xs = (self.txt, self.img), [x_txt, x_img]
        if mods is None:
            mods = [st.modulation(vec) for st in sts]
        else:
            mods = [list(mods[:4]), list(mods[4:])]

        def both(lin_of, ins, act=None):
            # the two streams' linears as one grouped GEMM launch (the 512-row text
            # stream alone would leave most SMs idle at small batch)
            return fp8_gemm_grouped2([(a8, a_s, lin_of(st).weight, lin_of(st).weight_scale, lin_of(st).bias)
                                      for st, (a8, a_s) in zip(sts, ins)], act=act)

        # norm + 1 x 128 quant in one pass, straight into the QKV GEMMs
        hs = [fused_rms_norm_modulate_quant(x, st.norm_w[0], m[0].contiguous(), cfg.eps)
              for st, x, m in zip(sts, xs, mods)]
        # attention output as each stream's out-projection input: text rows to one
        # code buffer, image rows to the other (no split copy, no separate quantiser)
        dev, D = x_txt.device, cfg.hidden
        codes = [(torch.empty(B, n, D, dtype=torch.float8_e4m3fn, device=dev),
                  torch.empty(B, n, D // 128, dtype=torch.float32, device=dev)) for n in (Nt, N - Nt)]
        freqs = (freqs_txt, freqs_img)
        if linear_prologue_ok([Nt, N - Nt], cfg.heads):
            # both QKV linears in one launch, P3 and the Q quantisation in its epilogue
            lin = [(h8, h_s, st.qkv.weight, st.qkv.weight_scale, st.qkv.bias, *f32_norms(st), fr, off, cfg.eps)
                   for st, (h8, h_s), fr, off in zip(sts, hs, freqs, (0, Nt))]
            attn_quant_out_from_linear(lin, cfg.heads, N, None, block_mask=None, qk_quant=cfg.qk_quant,
                                       pv_quant=cfg.pv_quant, granularity=cfg.granularity, regions=codes, split=Nt)
        else:
            qkvs = both(lambda st: st.qkv, hs)
            streams = [(qkvs[0], *f32_norms(self.txt), freqs_txt, 0, cfg.eps),
                       (qkvs[1], *f32_norms(self.img), freqs_img, Nt, cfg.eps)]
            joint_prologue_attention(streams, cfg, N, codes, split=Nt)
        attn = both(lambda st: st.proj, codes)
        xs = [fused_rms_norm_gate_residual(a, st.norm_w[1], m[1].contiguous(), x, cfg.eps)
              for st, a, x, m in zip(sts, attn, xs, mods)]
        hs = [fused_rms_norm_modulate_quant(x, st.norm_w[2], m[2].contiguous(), cfg.eps)
              for st, x, m in zip(sts, xs, mods)]
        gs = both(lambda st: st.mlp_in, hs, act=L.ACT_GELU_TANH)   # GELU(tanh) + requant epilogue
        fs = both(lambda st: st.mlp_out, gs)
        outs = [fused_rms_norm_gate_residual(f, st.norm_w[3], m[3].contiguous(), x, cfg.eps)
                for st, f, x, m in zip(sts, fs, xs, mods)]
        return outs[0], outs[1]


class SingleStreamBlock(nn.Module):
    """Single-stream block over the joint sequence: one linear (D -> 3D + rD)
    feeding attention and the MLP, one linear (D + rD -> D) for both outputs."""

    def __init__(self, cfg: DiTConfig, gen, device):
        super().__init__()
        self.cfg = cfg
        D, R = cfg.hidden, cfg.mlp_ratio
        self.adaln = nn.Linear(D, 2 * D, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            self.adaln.weight.copy_(_rand((2 * D, D), gen, device, 0.02))
            self.adaln.bias.copy_(_rand((2 * D,), gen, device, 0.02))
        self.norm_w = nn.ParameterList(
            [nn.Parameter(_rand((D,), gen, device, 0.05, 1.0), requires_grad=False) for _ in range(2)])
        self.q_norm = nn.Parameter(_rand((HEAD_DIM,), gen, device, 0.05, 1.0), requires_grad=False)
        self.k_norm = nn.Parameter(_rand((HEAD_DIM,), gen, device, 0.05, 1.0), requires_grad=False)
        # linear1 rows: [qkv (3D) | mlp_in (R D)]; linear2 columns: [attn (D) | mlp (R D)]
        self.linear1 = random_fp8_linear(3 * D + R * D, D, gen, device)
        self.linear2 = random_fp8_linear(D, D + R * D, gen, device)

    def forward(self, x: Tensor, vec: Tensor, freqs: Tensor, mods: Tensor | None = None) -> Tensor:
        """x (B, L, D) bf16; vec (B, D); freqs (B, L, 64, 2, 2) fp32; mods: the
        modulation (scale, gate) precomputed as (2, B, D), else computed from vec."""
        cfg = self.cfg
        B, N, D = x.shape
        if mods is None:
            scale, gate = self.adaln(torch.nn.functional.silu(vec)).chunk(2, dim=-1)
        else:
            scale, gate = mods[0], mods[1]
        a8, a_s = fused_rms_norm_modulate_quant(x, self.norm_w[0], scale.contiguous(), cfg.eps)
        w, ws = self.linear1.weight, self.linear1.weight_scale
        n_qkv = 3 * D
        # linear2's input [attention | MLP] as 1 x 128 codes: the GELU GEMM and the
        # attention write their halves of the same rows in place
        W = self.linear2.weight.shape[1]
        cat8 = torch.empty(B, N, W, dtype=torch.float8_e4m3fn, device=x.device)
        cat_s = torch.empty(B, N, W // 128, dtype=torch.float32, device=x.device)
        fp8_gemm_gelu_tanh_quant(a8, a_s, w[n_qkv:], ws[n_qkv // 128:], out=(cat8[..., D:], cat_s[..., D // 128:]))
        region = [(cat8[..., :D], cat_s[..., :D // 128])]
        if linear_prologue_ok([N], cfg.heads):
            # the QKV rows of linear1 with P3 and the Q quantisation in the GEMM epilogue
            lin = [(a8, a_s, w[:n_qkv], ws[: n_qkv // 128], None, *f32_norms(self), freqs, 0, cfg.eps)]
            attn_quant_out_from_linear(lin, cfg.heads, N, None, block_mask=None, qk_quant=cfg.qk_quant,
                                       pv_quant=cfg.pv_quant, granularity=cfg.granularity, regions=region)
        else:
            qkv = fp8_gemm_blockwise(a8, a_s, w[:n_qkv], ws[: n_qkv // 128], output_dtype=torch.bfloat16)
            joint_prologue_attention([(qkv, *f32_norms(self), freqs, 0, cfg.eps)], cfg, N, region)
        y = fp8_gemm_blockwise(cat8, cat_s, self.linear2.weight, self.linear2.weight_scale,
                               output_dtype=torch.bfloat16)
        return fused_rms_norm_gate_residual(y, self.norm_w[1], gate.contiguous(), x, cfg.eps)


def timestep_embedding(t: Tensor, dim: int, max_period: float = 10000.0) -> Tensor:
    """Sinusoidal embedding of t in [0, 1] (scaled by 1000), (B, dim) fp32."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = (t.float() * 1000.0)[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


class DiT(nn.Module):
    """Rectified-flow DiT: patch tokens + text tokens -> velocity of the patch tokens."""

    def __init__(self, cfg: DiTConfig, seed: int = 0, device="cuda"):
        super().__init__()
        self.cfg = cfg
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed)
        D = cfg.hidden
        if D != HEAD_DIM * cfg.heads:
            raise ValueError(f"hidden {D} must equal heads x {HEAD_DIM}")
        self.img_in = nn.Linear(cfg.patch_dim, D, device=dev, dtype=torch.bfloat16)
        self.time_in1 = nn.Linear(cfg.time_dim, D, device=dev, dtype=torch.bfloat16)
        self.time_in2 = nn.Linear(D, D, device=dev, dtype=torch.bfloat16)
        self.final_adaln = nn.Linear(D, D, device=dev, dtype=torch.bfloat16)
        self.final_out = nn.Linear(D, cfg.patch_dim, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            for lin in (self.img_in, self.time_in1, self.time_in2, self.final_adaln, self.final_out):
                lin.weight.copy_(_rand(tuple(lin.weight.shape), gen, dev, 0.02))
                lin.bias.zero_()
        self.final_norm = nn.Parameter(_rand((D,), gen, dev, 0.05, 1.0), requires_grad=False)
        self.double_blocks = nn.ModuleList([DoubleStreamBlock(cfg, gen, dev) for _ in range(cfg.n_double)])
        self.single_blocks = nn.ModuleList([SingleStreamBlock(cfg, gen, dev) for _ in range(cfg.n_single)])
        self.register_buffer("freqs_img", image_freqs(cfg, dev), persistent=False)
        self.register_buffer("freqs_txt", text_freqs(cfg, dev), persistent=False)
        self.register_buffer("freqs_all", torch.cat([self.freqs_txt, self.freqs_img], dim=0), persistent=False)
        self._freqs_cache: dict[int, tuple[Tensor, Tensor, Tensor]] = {}
        self._stack_modulation()

    def _stack_modulation(self) -> None:
        """Every block's adaLN linear as D x D chunks of one (C, D, D) weight stack
        (and a (C, 1, D) bias stack): chunk order = per double-stream block the text
        stream's four chunks then the image stream's, then per single-stream block
        (scale, gate).  The blocks' own adaLN parameters become views of the stacks
        (same values, no second copy), so ``modulations`` computes all of them with
        one batched GEMM per forward instead of a SiLU, a GEMV and the chunk copies
        per block (about 290 small launches of a 57-block step).  Weights loaded in
        place land in the stacks through the views; parameters that are replaced or
        moved (``load_state_dict(..., assign=True)``, ``.to()``) no longer view them,
        which ``modulations`` detects by address and restacks."""
        lins = [st.adaln for blk in self.double_blocks for st in (blk.txt, blk.img)]
        lins += [blk.adaln for blk in self.single_blocks]
        D = self.cfg.hidden
        chunks = [lin.weight.shape[0] // D for lin in lins]
        C = sum(chunks)
        dev = lins[0].weight.device if lins else self.freqs_img.device
        w = torch.empty(C, D, D, dtype=torch.bfloat16, device=dev)
        b = torch.empty(C, 1, D, dtype=torch.bfloat16, device=dev)
        c0 = 0
        with torch.no_grad():
            for lin, n in zip(lins, chunks):
                w[c0:c0 + n].copy_(lin.weight.view(n, D, D))
                b[c0:c0 + n].copy_(lin.bias.view(n, 1, D))
                lin.weight = nn.Parameter(w[c0:c0 + n].view(n * D, D), requires_grad=False)
                lin.bias = nn.Parameter(b[c0:c0 + n].view(n * D), requires_grad=False)
                c0 += n
        self.mod_w, self.mod_b = w, b
        self._mod_lins = lins
        self._mod_key = self._modulation_key()

    def _modulation_key(self) -> list[tuple[int, int]]:
        return [(lin.weight.data_ptr(), lin.bias.data_ptr()) for lin in self._mod_lins]

    def modulations(self, vec: Tensor) -> Tensor:
        """adaLN(SiLU(vec)) of every block at once: (C, B, D) bf16, chunk c of the
        stacks of ``_stack_modulation`` (one batched GEMM with the bias as its C input)."""
        if self._modulation_key() != self._mod_key:
            self._stack_modulation()
        C, D = self.mod_w.shape[0], self.cfg.hidden
        s = torch.nn.functional.silu(vec).unsqueeze(0).expand(C, vec.shape[0], D)
        return torch.baddbmm(self.mod_b, s, self.mod_w.transpose(1, 2))

    @torch.no_grad()
    def forward(self, img: Tensor, txt: Tensor, t: Tensor) -> Tensor:
        """img (B, img_tokens, patch_dim) bf16, txt (B, txt_tokens, hidden) bf16, t (B,) in [0, 1]."""
        cfg = self.cfg
        vec = self.time_in2(torch.nn.functional.silu(self.time_in1(
            timestep_embedding(t, cfg.time_dim).to(torch.bfloat16))))
        x_img = self.img_in(img).contiguous()
        x_txt = txt.contiguous()
        B = img.shape[0]
        if B not in self._freqs_cache:
            self._freqs_cache[B] = tuple(batch_freqs(f, B) for f in (self.freqs_txt, self.freqs_img, self.freqs_all))
        f_txt, f_img, f_all = self._freqs_cache[B]
        mods = self.modulations(vec)
        c = 0
        for blk in self.double_blocks:
            x_txt, x_img = blk(x_txt, x_img, vec, f_txt, f_img, mods=mods[c:c + 8])
            c += 8
        x = torch.cat([x_txt, x_img], dim=1)
        for blk in self.single_blocks:
            x = blk(x, vec, f_all, mods=mods[c:c + 2])
            c += 2
        x_img = x[:, cfg.txt_tokens:].contiguous()
        scale = self.final_adaln(torch.nn.functional.silu(vec)).contiguous()
        h = fused_rms_norm_modulate(x_img, self.final_norm, scale, cfg.eps)
        return self.final_out(h)


class EulerStepGraph:
    """One Euler step of ``model`` for a fixed batch shape, captured once as a CUDA
    graph and replayed: the ~1350 kernel launches of a step cost one graph launch
    (the kernels read their tensor maps and arguments from the captured launch
    parameters; the host side of the library is not re-run).  Each call copies
    x / txt into the static input buffers and the step's sigmas into device
    scalars, replays, and returns the static output buffer, which the next call
    overwrites.  Results are bit-identical to ``euler_step``."""

    def __init__(self, model: DiT, x: Tensor, txt: Tensor, warmup: int = 2):
        self.model = model
        dev = x.device
        self.x = x.detach().clone()
        self.txt = txt.detach().clone()
        self.t = torch.zeros(x.shape[0], dtype=torch.float32, device=dev)
        self.dt = torch.zeros(1, dtype=torch.float32, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):  # first launches set kernel attributes outside the capture
                self._step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._step()

    @torch.no_grad()
    def _step(self) -> Tensor:
        v = self.model(self.x, self.txt, self.t)
        return (self.x.float() + self.dt * v.float()).to(self.x.dtype)

    def __call__(self, x: Tensor, txt: Tensor, sigma: float, sigma_next: float) -> Tensor:
        if x.data_ptr() != self.x.data_ptr():
            self.x.copy_(x, non_blocking=True)
        if txt.data_ptr() != self.txt.data_ptr():
            self.txt.copy_(txt, non_blocking=True)
        self.t.fill_(sigma)
        self.dt.fill_(sigma_next - sigma)
        self.graph.replay()
        return self.out


@torch.no_grad()
def euler_step(model: DiT, x: Tensor, txt: Tensor, sigma: float, sigma_next: float) -> Tensor:
    """One rectified-flow Euler step: x + (sigma_next - sigma) * v(x, sigma)."""
    t = torch.full((x.shape[0],), sigma, device=x.device, dtype=torch.float32)
    v = model(x, txt, t)
    return (x.float() + (sigma_next - sigma) * v.float()).to(x.dtype)


def sigmas(steps: int) -> list[float]:
    """Linear flow-matching schedule from 1 (noise) to 0 (data)."""
    return [1.0 - i / steps for i in range(steps + 1)]


@torch.no_grad()
def euler_denoise(model: DiT, x: Tensor, txt: Tensor, steps: int = 28, graph: bool = False) -> Tensor:
    """``steps`` Euler steps; ``graph`` replays one captured CUDA graph per step."""
    s = sigmas(steps)
    if graph:
        g = EulerStepGraph(model, x, txt)
        for i in range(steps):
            x = g(x, txt, s[i], s[i + 1])
        return x.clone()
    for i in range(steps):
        x = euler_step(model, x, txt, s[i], s[i + 1])
    return x


def flops_per_sample_step(cfg: DiTConfig) -> float:
    """Algorithmic FLOPs of one forward of one sample: block linears + attention."""
    D, R, N = cfg.hidden, cfg.mlp_ratio, cfg.tokens
    lin_double = 2 * (3 + 1 + 2 * R) * D * D * N      # both streams together cover N tokens
    lin_single = 2 * ((3 + R) * D * D + (1 + R) * D * D) * N
    attn = 4 * N * N * D
    return cfg.n_double * (lin_double + attn) + cfg.n_single * (lin_single + attn)


# ------------------------------------------------------------------ video DiT (Ulysses)
@dataclass
class VideoDiTConfig:
    hidden: int = 5120
    heads: int = 40
    ffn: int = 13824
    n_blocks: int = 40
    grid: tuple[int, int, int] = (21, 30, 52)   # latent frames x patch rows x patch cols
    patch_dim: int = 64                         # 16 latent channels x 1 x 2 x 2
    txt_tokens: int = 512
    time_dim: int = 256
    rope_axes: tuple[int, int, int] = (44, 42, 42)
    rope_theta: float = 10000.0
    eps: float = 1e-5
    qk_quant: str = "int8"
    pv_quant: str = "bf16"
    granularity: str = "per_block"

    @property
    def tokens(self) -> int:
        t, h, w = self.grid
        return t * h * w


def video_freqs(cfg: VideoDiTConfig, device, start: int = 0, count: int | None = None) -> Tensor:
    """3-D RoPE rotations of video tokens [start, start + count) of the (t, h, w)
    grid, (count, head_dim/2, 2, 2) fp32."""
    t, h, w = cfg.grid
    count = cfg.tokens - start if count is None else count
    idx = torch.arange(start, start + count, device=device)
    pos = (idx // (h * w), (idx // w) % h, idx % w)
    parts = [rope_embed(p, d, cfg.rope_theta) for p, d in zip(pos, cfg.rope_axes)]
    return torch.cat(parts, dim=-3).contiguous()


class VideoBlock(nn.Module):
    """Video DiT block: self-attention over the (sequence-sharded) video tokens,
    cross-attention to the text tokens, GELU(tanh) FFN; every linear FP8."""

    def __init__(self, cfg: VideoDiTConfig, gen, device):
        super().__init__()
        self.cfg = cfg
        D = cfg.hidden
        self.adaln = nn.Linear(D, 4 * D, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            self.adaln.weight.copy_(_rand((4 * D, D), gen, device, 0.02))
            self.adaln.bias.copy_(_rand((4 * D,), gen, device, 0.02))
        self.norm_w = nn.ParameterList(
            [nn.Parameter(_rand((D,), gen, device, 0.05, 1.0), requires_grad=False) for _ in range(6)])
        self.cross_gate = nn.Parameter(_rand((1, D), gen, device, 0.5), requires_grad=False)
        self.q_norm = nn.Parameter(_rand((HEAD_DIM,), gen, device, 0.05, 1.0), requires_grad=False)
        self.k_norm = nn.Parameter(_rand((HEAD_DIM,), gen, device, 0.05, 1.0), requires_grad=False)
        self.qkv = random_fp8_linear(3 * D, D, gen, device)
        self.proj = random_fp8_linear(D, D, gen, device)
        self.cq = random_fp8_linear(D, D, gen, device)
        self.ckv = random_fp8_linear(2 * D, D, gen, device)
        self.co = random_fp8_linear(D, D, gen, device)
        self.ffn_in = random_fp8_linear(cfg.ffn, D, gen, device)
        self.ffn_out = random_fp8_linear(D, cfg.ffn, gen, device)

    def forward(self, x: Tensor, vec: Tensor, txt: Tensor, freqs: Tensor, group=None, head_groups: int = 1) -> Tensor:
        """x (1, L/P, D) bf16: this rank's tokens; vec (1, D); txt (1, 512, D); freqs (1, L/P, 64, 2, 2);
        head_groups: how many head groups pipeline the Ulysses exchange with the attention."""
        from .ulysses import ulysses_attention_codes

        cfg = self.cfg
        _, Ls, D = x.shape
        H = cfg.heads
        m = [c.contiguous() for c in self.adaln(torch.nn.functional.silu(vec)).chunk(4, dim=-1)]
        # ---- self-attention (Ulysses: sequence -> head all-to-all around the kernel)
        h8, h_s = fused_rms_norm_modulate_quant(x, self.norm_w[0], m[0], cfg.eps)
        qkv = gemm_bf16(h8, h_s, self.qkv)
        q, k, v = fused_qkv_postprocess(qkv, *f32_norms(self), freqs, H, HEAD_DIM, cfg.eps)

        def attn_codes(qh, kh, vh):
            # the output projection's 1 x 128 e4m3 input, written by the attention kernel
            _, Hl, L, _ = qh.shape
            c8 = torch.empty(L, Hl * HEAD_DIM, dtype=torch.uint8, device=qh.device)
            cs = torch.empty(L, Hl, dtype=torch.float32, device=qh.device)
            attn_forward_quant_out(qh, kh, vh, None, block_mask=None, qk_quant=cfg.qk_quant,
                                   pv_quant=cfg.pv_quant, granularity=cfg.granularity, regions=[(c8, cs)])
            return c8, cs

        o8, o_s = ulysses_attention_codes(q[0], k[0], v[0], attn_codes, group, head_groups)  # (L/P, D), (L/P, D/128)
        a = gemm_bf16(o8.view(torch.float8_e4m3fn).unsqueeze(0), o_s.unsqueeze(0), self.proj)
        x = fused_rms_norm_gate_residual(a, self.norm_w[1], m[1], x, cfg.eps)
        # ---- cross-attention to the text (replicated on every rank; 512 keys, bf16 SDPA)
        zero = torch.zeros_like(m[0])
        c8, c_s = fused_rms_norm_modulate_quant(x, self.norm_w[2], zero, cfg.eps)
        qc = gemm_bf16(c8, c_s, self.cq).view(1, Ls, H, HEAD_DIM).transpose(1, 2)
        kv = linear_bf16(txt, self.ckv).view(1, -1, 2, H, HEAD_DIM)
        kc, vc = kv[:, :, 0].transpose(1, 2), kv[:, :, 1].transpose(1, 2)
        oc = torch.nn.functional.scaled_dot_product_attention(qc, kc, vc)
        ac = linear_bf16(oc.transpose(1, 2).reshape(1, Ls, D).contiguous(), self.co)
        x = fused_rms_norm_gate_residual(ac, self.norm_w[3], self.cross_gate.expand(1, D).contiguous(), x, cfg.eps)
        # ---- FFN
        f8, f_s = fused_rms_norm_modulate_quant(x, self.norm_w[4], m[2], cfg.eps)
        f = mlp_fp8_q(f8, f_s, self.ffn_in, self.ffn_out)
        return fused_rms_norm_gate_residual(f, self.norm_w[5], m[3], x, cfg.eps)


class VideoDiT(nn.Module):
    """14B-class video DiT, sequence-parallel over a process group (Ulysses)."""

    def __init__(self, cfg: VideoDiTConfig, seed: int = 0, device="cuda", group=None, head_groups: int = 1):
        """head_groups > 1 pipelines each Ulysses exchange with the attention by head
        groups (``ulysses_attention_codes``); the output is the same for every value."""
        super().__init__()
        import torch.distributed as dist

        self.cfg = cfg
        self.group = group
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed)   # identical weights on every rank
        D = cfg.hidden
        if D != HEAD_DIM * cfg.heads:
            raise ValueError(f"hidden {D} must equal heads x {HEAD_DIM}")
        P = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        if cfg.tokens % P or cfg.heads % P:
            raise ValueError(f"{cfg.tokens} tokens / {cfg.heads} heads do not split over {P} ranks")
        self.P, self.rank = P, rank
        self.local_tokens = cfg.tokens // P
        if cfg.heads % (P * head_groups):
            raise ValueError(f"{cfg.heads} heads do not split into {head_groups} groups over {P} ranks")
        self.head_groups = head_groups
        self.img_in = nn.Linear(cfg.patch_dim, D, device=dev, dtype=torch.bfloat16)
        self.time_in1 = nn.Linear(cfg.time_dim, D, device=dev, dtype=torch.bfloat16)
        self.time_in2 = nn.Linear(D, D, device=dev, dtype=torch.bfloat16)
        self.final_adaln = nn.Linear(D, D, device=dev, dtype=torch.bfloat16)
        self.final_out = nn.Linear(D, cfg.patch_dim, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            for lin in (self.img_in, self.time_in1, self.time_in2, self.final_adaln, self.final_out):
                lin.weight.copy_(_rand(tuple(lin.weight.shape), gen, dev, 0.02))
                lin.bias.zero_()
        self.final_norm = nn.Parameter(_rand((D,), gen, dev, 0.05, 1.0), requires_grad=False)
        self.blocks = nn.ModuleList([VideoBlock(cfg, gen, dev) for _ in range(cfg.n_blocks)])
        f = video_freqs(cfg, dev, rank * self.local_tokens, self.local_tokens)
        self.register_buffer("freqs_local", f.unsqueeze(0).contiguous(), persistent=False)

    @torch.no_grad()
    def forward(self, x_local: Tensor, txt: Tensor, t: Tensor) -> Tensor:
        """x_local (1, L/P, patch_dim): this rank's latent tokens; txt (1, 512, D); t (1,)."""
        cfg = self.cfg
        vec = self.time_in2(torch.nn.functional.silu(self.time_in1(
            timestep_embedding(t, cfg.time_dim).to(torch.bfloat16))))
        x = self.img_in(x_local).contiguous()
        for blk in self.blocks:
            x = blk(x, vec, txt, self.freqs_local, self.group, self.head_groups)
        scale = self.final_adaln(torch.nn.functional.silu(vec)).contiguous()
        return self.final_out(fused_rms_norm_modulate(x, self.final_norm, scale, cfg.eps))


def video_flops_per_step(cfg: VideoDiTConfig) -> float:
    """Algorithmic FLOPs of one forward (one sample): linears, self- and cross-attention."""
    D, F, L, T = cfg.hidden, cfg.ffn, cfg.tokens, cfg.txt_tokens
    lin = 2 * L * (4 * D * D + 2 * D * D + 2 * D * F) + 2 * T * 2 * D * D
    return cfg.n_blocks * (lin + 4 * L * L * D + 4 * L * T * D)
