"""h3q.dit -- one DiT transformer block on the library: the reference's call sites of the hot-path ops
(Dit::run_block, dit.rs:969-1021).

The reference's block, for the packed token stream x [S, C] (bf16) and its adaLN tables (f32 [R, C] rows selected
per token by idx [S]):

    n1  = rms_modulate(x, norm1, eps, scale_msa, shift_msa, idx)            dit.rs:981
    qkv = qkv.forward_raw(n1)                 gemm_s8 with ConvRot           dit.rs:985
    att = attend(qkv, q_norm, k_norm, rope)   q/k RMSNorm + RoPE + int8 attention, dit.rs:987
    o   = out.forward_raw(att)                gemm_s8 with ConvRot           dit.rs:992
    x   = gate_add(x, o, gate_msa, idx)                                        dit.rs:994
    n2  = rms_modulate(x, norm2, eps, scale_mlp, shift_mlp, idx)            dit.rs:997
    h   = fc1.run_swiglu(n2)                  gemm_s8, SwiGLU on (gate, up) row pairs, dit.rs:1008
    m   = fc2.run(h)                          gemm_s8 with ConvRot           dit.rs:1009
    x   = gate_add(x, m, gate_mlp, idx)                                        dit.rs:1017

`run_block_ops` issues exactly those calls through the library.  `run_block` is the same block with the fusions the
library offers: the modulation feeds the quantizer directly (h3q_rms_modulate_quant: no bf16 round trip of n1 / n2),
the SwiGLU runs in the fc1 GEMM's epilogue, and each gate_add runs in the out / fc2 GEMM's epilogue (the gated
residual epilogue).  Both give the same bits.  The adaLN projection that produces the tables (dit.rs:976) and the
block's LoRA handling stay with the caller.  ControlNet blocks run the same block (control.rs:180).  Above a 1.5 GB
qkv the reference projects and attends head group by head group (attn_groups / attend_grouped, dit.rs:762-801).
"""
from __future__ import annotations

from dataclasses import dataclass

from . import (EPI_GATE_RESID, EPI_LINEAR, EPI_SWIGLU_PAIRS, attend_qkv, attention_qkv, gate_add, gemm_s8,
               gemm_s8_quantized, qk_norm_rope, quant_rows, rms_modulate, rms_modulate_quant)

ATTN_QKV_BUDGET = 1_500_000_000   # bytes of bf16 qkv above which the reference splits the attention (dit.rs:361)


@dataclass
class Linear:
    """An int8 ConvRot layer: weight int8 [N, K], per-row scale f32 [N] (or one), bias f32 [N] or None."""
    w: object
    ws: object
    bias: object = None


@dataclass
class Block:
    """A block's weights (dit.rs Block): fc1 holds (gate, up) row pairs, as QLinear::interleave_swiglu stores them."""
    qkv: Linear
    out: Linear
    fc1: Linear
    fc2: Linear
    norm1: object    # bf16 [C]
    norm2: object    # bf16 [C]
    q_norm: object   # bf16 [128]
    k_norm: object   # bf16 [128]
    heads: int
    eps: float = 1e-6


@dataclass
class StepCtx:
    """Per-step inputs of a block (dit.rs StepCtx and the adaLN tables): f32 [R, C] tables, the table row of each
    token idx [S] (int32 / uint32), and the rope table f32 [2, S, rot / 2]."""
    shift_msa: object
    scale_msa: object
    gate_msa: object
    shift_mlp: object
    scale_mlp: object
    gate_mlp: object
    idx: object
    rope: object
    rot: int
    flags: int = 0


def attn_groups(tokens: int, heads: int, hidden: int, override: int | None = None) -> int:
    """Dit::attn_groups (dit.rs:762-773): 1 while the bf16 qkv (3 * tokens * hidden * 2 bytes) fits the budget,
    else the smallest divisor of heads that is at least the number of budgets it needs.  override plays the
    H3_ATTN_GROUPS variable: a divisor of heads is taken as is, anything else gives 1."""
    if override is not None:
        return override if override >= 1 and heads % override == 0 else 1
    qkv_bytes = 3 * tokens * hidden * 2
    if qkv_bytes <= ATTN_QKV_BUDGET:
        return 1
    want = -(-qkv_bytes // ATTN_QKV_BUDGET)
    return next((g for g in range(want, heads + 1) if heads % g == 0), heads)


def attend_grouped(n1, b: Block, cx: StepCtx, groups: int):
    """Dit::attend_grouped (dit.rs:778-801): the qkv projection and the attention `groups` head groups at a time,
    so that no more than a group's q, k and v exist at once.  Per group g: the q, k and v row blocks of the qkv
    weight (rows g w .. (g + 1) w of each third, w = heads / groups * 128) through gemm_s8, q / k RMSNorm + RoPE,
    then attention_qkv with V at column 0 of its own block; the groups' outputs side by side.  Every output column
    of the GEMM and every head of the attention is computed on its own here, so the result has the bits of the
    ungrouped qkv GEMM + attend_qkv."""
    import torch
    h, d = b.heads, 128
    inner = h * d
    hg = h // groups
    w = hg * d

    def proj(base: int, g: int):
        r0 = base + g * w
        ws = b.qkv.ws if b.qkv.ws.numel() == 1 else b.qkv.ws[r0:r0 + w]
        bias = None if b.qkv.bias is None else b.qkv.bias[r0:r0 + w]
        return gemm_s8(n1, b.qkv.w[r0:r0 + w], ws, bias, swiglu=False, rotate=True)

    outs = []
    for g in range(groups):
        q = qk_norm_rope(proj(0, g), 0, hg, d, (b.q_norm, b.eps), cx.rope, cx.rot)
        k = qk_norm_rope(proj(inner, g), 0, hg, d, (b.k_norm, b.eps), cx.rope, cx.rot)
        vt = proj(2 * inner, g)
        outs.append(attention_qkv(q, k, vt, 0, cx.flags).reshape(n1.shape[0], w))
    return outs[0] if groups == 1 else torch.cat(outs, dim=1)


def run_block_ops(x, b: Block, cx: StepCtx, trace: dict | None = None, groups: int | None = None):
    """The block as the reference issues it (dit.rs:981-1017), one library call per reference call.  With a dict
    as trace, each intermediate is kept in it under the reference's name (n1, qkv, att, o, x1, n2, h, m, y).
    groups: the attention's head groups (attn_groups of the token count when None); above 1 the qkv projection
    and the attention run group by group (attend_grouped) and trace holds no qkv."""
    n1 = rms_modulate(x, b.norm1, b.eps, cx.scale_msa, cx.shift_msa, cx.idx)
    if groups is None:
        groups = attn_groups(x.shape[0], b.heads, x.shape[1])
    if groups > 1:
        qkv = None
        att = attend_grouped(n1, b, cx, groups)
    else:
        qkv = gemm_s8(n1, b.qkv.w, b.qkv.ws, b.qkv.bias, swiglu=False, rotate=True)
        att = attend_qkv(qkv, b.heads, (b.q_norm, b.k_norm), b.eps, cx.rope, cx.rot, cx.flags)
    o = gemm_s8(att, b.out.w, b.out.ws, b.out.bias, swiglu=False, rotate=True)
    x1 = gate_add(x, o, cx.gate_msa, cx.idx)
    n2 = rms_modulate(x1, b.norm2, b.eps, cx.scale_mlp, cx.shift_mlp, cx.idx)
    h = gemm_s8(n2, b.fc1.w, b.fc1.ws, b.fc1.bias, swiglu=True, rotate=True)
    m = gemm_s8(h, b.fc2.w, b.fc2.ws, b.fc2.bias, swiglu=False, rotate=True)
    y = gate_add(x1, m, cx.gate_mlp, cx.idx)
    if trace is not None:
        trace.update(n1=n1, qkv=qkv, att=att, o=o, x1=x1, n2=n2, h=h, m=m, y=y)
    return y


def run_block(x, b: Block, cx: StepCtx):
    """The block with the library's fusions (module docstring); the same bits as run_block_ops."""
    q1, s1 = rms_modulate_quant(x, b.norm1, b.eps, cx.scale_msa, cx.shift_msa, cx.idx)
    qkv = gemm_s8_quantized(q1, s1, b.qkv.w, b.qkv.ws, b.qkv.bias, EPI_LINEAR)
    att = attend_qkv(qkv, b.heads, (b.q_norm, b.k_norm), b.eps, cx.rope, cx.rot, cx.flags)
    qa, sa = quant_rows(att, True)
    x = gemm_s8_quantized(qa, sa, b.out.w, b.out.ws, b.out.bias, EPI_GATE_RESID, gate=cx.gate_msa,
                          gate_idx=cx.idx, resid=x)
    q2, s2 = rms_modulate_quant(x, b.norm2, b.eps, cx.scale_mlp, cx.shift_mlp, cx.idx)
    h = gemm_s8_quantized(q2, s2, b.fc1.w, b.fc1.ws, b.fc1.bias, EPI_SWIGLU_PAIRS)
    qh, sh = quant_rows(h, True)
    return gemm_s8_quantized(qh, sh, b.fc2.w, b.fc2.ws, b.fc2.bias, EPI_GATE_RESID, gate=cx.gate_mlp,
                             gate_idx=cx.idx, resid=x)


__all__ = ["Linear", "Block", "StepCtx", "attn_groups", "attend_grouped", "run_block", "run_block_ops"]
