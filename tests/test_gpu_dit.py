"""GPU tests of a whole DiT block on the library (h3q.dit, Dit::run_block, dit.rs:969-1021): the fused block (the
modulation feeding the quantizer, SwiGLU and the gated residuals in the GEMM epilogues) gives the same bits as the
reference's op-by-op sequence, and both match the oracle's composition of the same steps within the attention's
tolerance."""
import numpy as np
import pytest
import torch

import h3q
from h3q import dit as D
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _inputs(seed, S, H, F, R=3, rot=96):
    rng = np.random.default_rng(seed)
    C = H * 128
    x, norm1, scale_msa, shift_msa, idx = O.make_modulate_inputs(seed, S, C, R)
    _, norm2, scale_mlp, shift_mlp, _ = O.make_modulate_inputs(seed + 1, S, C, R)
    gate_msa = rng.uniform(0.0, 1.0, (R, C)).astype(np.float32)
    gate_mlp = rng.uniform(0.0, 1.0, (R, C)).astype(np.float32)
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


@pytest.mark.parametrize("S,H,F", [(384, 4, 1024), (250, 2, 512)])
def test_block_fused_equals_ops_and_oracle(cuda, S, H, F):
    inp = _inputs(S + H + F, S, H, F)
    x, blk, cx = _device(inp, H, cuda)
    fused = D.run_block(x, blk, cx)
    ops = D.run_block_ops(x, blk, cx)
    torch.cuda.synchronize()
    assert fused.shape == x.shape
    assert torch.equal(fused.view(torch.int16), ops.view(torch.int16))
    want = _oracle_block(inp, H)
    got = fused.view(torch.int16).cpu().numpy().view(np.uint16)
    assert O.max_abs_rel(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want)) < TOL
    assert h3q.device_status() == 0


def test_block_chain_is_deterministic(cuda):
    """Two blocks in a row (the second on the first's output) give the same bits on a second run."""
    S, H, F = 256, 2, 512
    x, blk, cx = _device(_inputs(5, S, H, F), H, cuda)
    y1 = D.run_block(D.run_block(x, blk, cx), blk, cx)
    y2 = D.run_block(D.run_block(x, blk, cx), blk, cx)
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    assert bool(torch.isfinite(y1.float()).all())
