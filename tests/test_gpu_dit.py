"""GPU tests of a whole DiT block on the library (h3q.dit, Dit::run_block, dit.rs:969-1021).

* The fused block gives the same bits as the op-by-op sequence. The fused block feeds the modulation into the
  quantizer and runs SwiGLU and the gated residuals in the GEMM epilogues.
* Every step of the op-by-op block matches its oracle step when that step is fed the GPU's own input:
  - the qkv, out and fc2 linears and the two gated residuals bit for bit;
  - fc1's SwiGLU output within the SwiGLU tolerance 1e-2, because the device uses __expf and the oracle expf;
  - the modulations as rms_modulate's own test allows, or bit for bit against the reference kernel when it is
    built;
  - the attention within its 1e-2.
* The whole block stays near the oracle's composition of the nine steps. The block quantizes four activations to
  int8. A code that flips because of the attention's deviation, or a last-bit rsqrt difference in a modulation,
  adds one unit of a weight row to the next output, so the end-to-end bound is looser than any single step's.
"""
import numpy as np
import pytest
import torch

import h3q
from h3q import dit as D
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_bits

pytestmark = pytest.mark.gpu
ATTN_TOL = 1e-2
SWIGLU_TOL = 1e-2
BLOCK_TOL = 5e-2


def _inputs(seed, S, H, F, rows=3, rot=96):
    rng = np.random.default_rng(seed)
    C = H * 128
    x, norm1, scale_msa, shift_msa, idx = O.make_modulate_inputs(seed, S, C, rows)
    _, norm2, scale_mlp, shift_mlp, _ = O.make_modulate_inputs(seed + 1, S, C, rows)
    gate_msa = rng.uniform(0.0, 1.0, (rows, C)).astype(np.float32)
    gate_mlp = rng.uniform(0.0, 1.0, (rows, C)).astype(np.float32)
    _, qw, kw, cs = O.make_rope_inputs(seed + 2, S, H, 128, rot)

    def lin(n, k):
        w = rng.integers(-127, 128, (n, k)).astype(np.int8)
        ws = rng.uniform(1e-3, 1e-2, n).astype(np.float32)
        b = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.normal(0, 0.02, n).astype(np.float32)))
        return w, ws, b
    lins = {"qkv": lin(3 * C, C), "out": lin(C, C), "fc1": lin(2 * F, C), "fc2": lin(C, F)}
    return dict(x=x, norm1=norm1, norm2=norm2, qw=qw, kw=kw, cs=cs, rot=rot, idx=idx, lins=lins,
                tables=dict(scale_msa=scale_msa, shift_msa=shift_msa, gate_msa=gate_msa, scale_mlp=scale_mlp,
                            shift_mlp=shift_mlp, gate_mlp=gate_mlp))


def _device(inp, H, dev):
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    L = {k: D.Linear(t(w), t(ws), t(b)) for k, (w, ws, b) in inp["lins"].items()}
    blk = D.Block(L["qkv"], L["out"], L["fc1"], L["fc2"], bf(inp["norm1"]), bf(inp["norm2"]), bf(inp["qw"]),
                  bf(inp["kw"]), H)
    tb = {k: t(v) for k, v in inp["tables"].items()}
    cx = D.StepCtx(tb["shift_msa"], tb["scale_msa"], tb["gate_msa"], tb["shift_mlp"], tb["scale_mlp"], tb["gate_mlp"],
                   t(inp["idx"].astype(np.int32)), t(inp["cs"]), inp["rot"])
    return bf(inp["x"]), blk, cx


def _oracle_block(inp, H, eps=1e-6):
    tb, L, idx = inp["tables"], inp["lins"], inp["idx"]
    n1 = O.rms_modulate(inp["x"], inp["norm1"], eps, tb["scale_msa"], tb["shift_msa"], idx)
    qkv = O.gemm_s8(n1, *L["qkv"], False, True)[0]
    att = O.attend_qkv(qkv, H, inp["qw"], inp["kw"], True, eps, inp["cs"], inp["rot"]).reshape(qkv.shape[0], -1)
    o = O.gemm_s8(att, *L["out"], False, True)[0]
    x1 = O.gate_add(inp["x"], o, 2, tb["gate_msa"], idx)
    n2 = O.rms_modulate(x1, inp["norm2"], eps, tb["scale_mlp"], tb["shift_mlp"], idx)
    h = O.gemm_s8(n2, *L["fc1"], True, True)[0]
    m = O.gemm_s8(h, *L["fc2"], False, True)[0]
    return O.gate_add(x1, m, 2, tb["gate_mlp"], idx)


def _check_modulate(got_t, x_t, w_t, scale_t, shift_t, idx_t, eps):
    got = bf16_bits(got_t)
    if R.available():
        want = bf16_bits(R.rms_modulate(x_t, w_t, eps, scale_t, shift_t, idx_t))
        assert np.array_equal(got, want)
        return
    want = O.rms_modulate(bf16_bits(x_t), bf16_bits(w_t), eps, scale_t.cpu().numpy(), shift_t.cpu().numpy(),
                          idx_t.cpu().numpy().astype(np.uint32))
    assert (got == want).mean() > 0.99
    assert O.max_abs_rel(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want)) <= 1e-2


@pytest.mark.parametrize("S,H,F", [(384, 4, 1024), (250, 2, 512)])
def test_block_fused_equals_ops_and_oracle(cuda, S, H, F):
    inp = _inputs(S + H + F, S, H, F)
    x, blk, cx = _device(inp, H, cuda)
    fused = D.run_block(x, blk, cx)
    tr = {}
    ops = D.run_block_ops(x, blk, cx, trace=tr)
    torch.cuda.synchronize()
    assert fused.shape == x.shape
    assert torch.equal(fused.view(torch.int16), ops.view(torch.int16))
    assert torch.equal(ops.view(torch.int16), tr["y"].view(torch.int16))

    L, tb, idx = inp["lins"], inp["tables"], inp["idx"]
    g = {k: bf16_bits(v) for k, v in tr.items()}
    _check_modulate(tr["n1"], x, blk.norm1, cx.scale_msa, cx.shift_msa, cx.idx, blk.eps)
    assert np.array_equal(g["qkv"], O.gemm_s8(g["n1"], *L["qkv"], False, True)[0])
    att = O.attend_qkv(g["qkv"], H, inp["qw"], inp["kw"], True, blk.eps, inp["cs"], inp["rot"]).reshape(S, -1)
    assert O.max_abs_rel(O.bf16_bits_to_f32(g["att"]), O.bf16_bits_to_f32(att)) < ATTN_TOL
    assert np.array_equal(g["o"], O.gemm_s8(g["att"], *L["out"], False, True)[0])
    assert np.array_equal(g["x1"], O.gate_add(inp["x"], g["o"], 2, tb["gate_msa"], idx))
    _check_modulate(tr["n2"], tr["x1"], blk.norm2, cx.scale_mlp, cx.shift_mlp, cx.idx, blk.eps)
    h = O.gemm_s8(g["n2"], *L["fc1"], True, True)[0]   # SwiGLU: __expf on the device, expf in the oracle
    assert (g["h"] == h).mean() > 0.99
    assert O.max_abs_rel(O.bf16_bits_to_f32(g["h"]), O.bf16_bits_to_f32(h)) < SWIGLU_TOL
    assert np.array_equal(g["m"], O.gemm_s8(g["h"], *L["fc2"], False, True)[0])
    assert np.array_equal(g["y"], O.gate_add(g["x1"], g["m"], 2, tb["gate_mlp"], idx))

    want = _oracle_block(inp, H)
    assert O.max_abs_rel(O.bf16_bits_to_f32(g["y"]), O.bf16_bits_to_f32(want)) < BLOCK_TOL
    assert h3q.device_status() == 0


def test_block_chain_is_deterministic(cuda):
    """Two blocks in a row (the second on the first's output) give the same bits on a second run."""
    S, H, F = 256, 2, 512
    x, blk, cx = _device(_inputs(5, S, H, F), H, cuda)
    y1 = D.run_block(D.run_block(x, blk, cx), blk, cx)
    y2 = D.run_block(D.run_block(x, blk, cx), blk, cx)
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    assert bool(torch.isfinite(y1.float()).all())


@pytest.mark.parametrize("groups", [2, 4])
def test_grouped_attention_equals_ungrouped(cuda, groups):
    """Dit::attend_grouped (dit.rs:778-801): the qkv projection and attention head group by head group give the
    bits of the whole qkv GEMM + attend_qkv, and the block run that way the bits of the fused block."""
    S, H, F = 300, 4, 512
    x, blk, cx = _device(_inputs(7 + groups, S, H, F), H, cuda)
    n1 = h3q.rms_modulate(x, blk.norm1, blk.eps, cx.scale_msa, cx.shift_msa, cx.idx)
    qkv = h3q.gemm_s8(n1, blk.qkv.w, blk.qkv.ws, blk.qkv.bias, swiglu=False, rotate=True)
    whole = h3q.attend_qkv(qkv, H, (blk.q_norm, blk.k_norm), blk.eps, cx.rope, cx.rot, cx.flags).reshape(S, -1)
    grouped = D.attend_grouped(n1, blk, cx, groups)
    assert torch.equal(grouped.view(torch.int16), whole.view(torch.int16))
    y = D.run_block_ops(x, blk, cx, groups=groups)
    assert torch.equal(y.view(torch.int16), D.run_block(x, blk, cx).view(torch.int16))
    assert h3q.device_status() == 0
