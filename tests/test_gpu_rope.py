"""GPU parity of qk_norm_rope (kernels.rs:86-126) and of the DiT attention step with it fused into the int8
attention's front end (dit.rs:741-757).

Bit-exact: h3q_qk_norm_rope against the reference's kernel compiled for sm_100a (same reduction order, hardware
rsqrtf, the same FMA contraction in the rotation); h3q_attend_qkv against h3q_qk_norm_rope + h3q_attention_qkv (the
fused front end produces the same codes, scales and K mean).  Against the CPU oracle (1 / sqrtf for rsqrtf): over
99% of the outputs identical, all within 1e-2; the attention step within the bf16 output contract (1e-2).
"""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_bits, bf16_tensor, t

pytestmark = pytest.mark.gpu

EPS = 1e-6
TOL = 1e-2

# (S, H, D, rot, norm weight, head stride factor): the DiT's q / k (D 128, rot 96), a full rotation, no rotation,
# D not a multiple of 32, the widest head, a VAE-like interleaved layout (head stride 3 D, rot 48); at D 128 every
# rot % 32 == 0 runs the pair layout, other rot % 8 == 0 the slice layout
CASES = [(300, 40, 128, 96, True, 1), (200, 2, 128, 128, False, 1), (1000, 24, 128, 0, True, 1),
         (33, 3, 80, 48, True, 1), (50, 4, 256, 128, True, 1), (77, 6, 64, 48, True, 3), (1, 1, 32, 32, False, 1),
         (150, 5, 128, 64, True, 1), (90, 3, 128, 32, True, 3), (120, 4, 128, 48, True, 1), (64, 2, 128, 8, False, 1)]


def _case(S, H, D, rot, use_w, hsf, seed):
    rng = np.random.default_rng(seed)
    width = 3 * H * D * hsf
    x = O.f32_to_bf16_bits((rng.standard_normal((S, width)) * (1 + 3 * rng.random((S, 1)))).astype(np.float32))
    w = O.f32_to_bf16_bits((1 + 0.2 * rng.standard_normal(D)).astype(np.float32)) if use_w else None
    cs = None
    if rot:
        ang = (100 * rng.random((S, rot // 2))).astype(np.float32)
        cs = O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.stack([np.cos(ang), np.sin(ang)]))).reshape(2, S, rot // 2)
    return x, w, cs


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("S,H,D,rot,use_w,hsf", CASES)
def test_qk_norm_rope_matches_reference_kernel(cuda, S, H, D, rot, use_w, hsf):
    x, w, cs = _case(S, H, D, rot, use_w, hsf, S + D)
    tx, tw = bf16_tensor(x, cuda), None if w is None else bf16_tensor(w, cuda)
    tcs = None if cs is None else t(np.ascontiguousarray(cs), cuda)
    col, hs = D * hsf, D * hsf
    for do_norm in (True, False):
        got = h3q.qk_norm_rope(tx, col, H, D, (tw, EPS) if do_norm else None, tcs, rot, head_stride=hs)
        want = R.qk_norm_rope(tx, col, hs, H, D, tw, EPS, do_norm, tcs, rot)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert h3q.device_status() == 0


@pytest.mark.parametrize("S,H,D,rot,use_w,hsf", CASES)
def test_qk_norm_rope_vs_oracle(cuda, S, H, D, rot, use_w, hsf):
    x, w, cs = _case(S, H, D, rot, use_w, hsf, 2 * S + D)
    tx, tw = bf16_tensor(x, cuda), None if w is None else bf16_tensor(w, cuda)
    tcs = None if cs is None else t(np.ascontiguousarray(cs), cuda)
    got = bf16_bits(h3q.qk_norm_rope(tx, 0, H, D, (tw, EPS), tcs, rot, head_stride=D * hsf))
    want = O.qk_norm_rope(x, 0, H, D, w, EPS, True, cs, rot, head_stride=D * hsf)
    assert (got == want).mean() > 0.99
    assert O.max_abs_rel(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want)) <= 1e-2
    # without the norm there is no rsqrtf: bit-exact
    got = bf16_bits(h3q.qk_norm_rope(tx, 0, H, D, None, tcs, rot, head_stride=D * hsf))
    want = O.qk_norm_rope(x, 0, H, D, None, EPS, False, cs, rot, head_stride=D * hsf)
    np.testing.assert_array_equal(got, want)


def test_qk_norm_rope_reference_known_answer(cuda):
    """portable/kernels.rs:357-380 on the device: zero angles over rot = 2 leave [[1, 2], [3, 4]] unchanged."""
    x = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device=cuda).to(torch.bfloat16)
    cs = torch.stack([torch.ones(2, 1), torch.zeros(2, 1)]).to(cuda)
    y = h3q.qk_norm_rope(x, 0, 1, 2, None, cs, 2)
    assert y.float().reshape(-1).tolist() == [1.0, 2.0, 3.0, 4.0]


@pytest.mark.parametrize("flags", [0, 1, 2, 3])
@pytest.mark.parametrize("S,H,rot,norm", [(300, 4, 96, True), (1000, 3, 128, True), (2053, 2, 96, False),
                                          (129, 2, 0, True), (4000, 1, 48, True), (500, 2, 64, True),
                                          (257, 3, 32, True), (1100, 9, 96, True)])
def test_attend_qkv_equals_unfused(cuda, S, H, rot, norm, flags):
    """The fused front end gives the bits of qk_norm_rope -> attention_qkv (dit.rs:748-750)."""
    qkv, qw, kw, cs = O.make_rope_inputs(S + H, S, H, 128, max(rot, 8))
    tqkv = bf16_tensor(qkv, cuda)
    tqw, tkw, tcs = bf16_tensor(qw, cuda), bf16_tensor(kw, cuda), t(cs, cuda)
    rope = tcs if rot else None
    inner = H * 128
    out = h3q.attend_qkv(tqkv, H, (tqw, tkw) if norm else None, EPS, rope, rot, flags)
    q = h3q.qk_norm_rope(tqkv, 0, H, 128, (tqw, EPS) if norm else None, rope, rot)
    k = h3q.qk_norm_rope(tqkv, inner, H, 128, (tkw, EPS) if norm else None, rope, rot)
    want = h3q.attention_qkv(q, k, tqkv, 2 * inner, flags).reshape(S, inner)
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    assert h3q.device_status() == 0


@pytest.mark.parametrize("S,H,flags", [(300, 2, 0), (260, 1, 3)])
def test_attend_qkv_vs_oracle(cuda, S, H, flags):
    qkv, qw, kw, cs = O.make_rope_inputs(7 * S, S, H, 128, 96)
    out = h3q.attend_qkv(bf16_tensor(qkv, cuda), H, (bf16_tensor(qw, cuda), bf16_tensor(kw, cuda)), EPS,
                         t(cs, cuda), 96, flags)
    ref = O.attend_qkv(qkv, H, qw, kw, True, EPS, cs, 96, flags)
    err = O.max_abs_rel(O.bf16_bits_to_f32(bf16_bits(out)).reshape(S, H, 128), O.bf16_bits_to_f32(ref))
    assert err <= TOL, err


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
def test_attend_qkv_vs_reference_chain(cuda):
    """The reference's own chain on the device: its qk_norm_rope, then (with h3q's bit-exact K mean and QuantHeads,
    which equal its ColMean / QuantHeads up to ColMean's atomic order) attn_qk8."""
    S, H, rot = 600, 2, 96
    qkv, qw, kw, cs = O.make_rope_inputs(17, S, H, 128, rot)
    tqkv, tqw, tkw, tcs = bf16_tensor(qkv, cuda), bf16_tensor(qw, cuda), bf16_tensor(kw, cuda), t(cs, cuda)
    inner = H * 128
    out = h3q.attend_qkv(tqkv, H, (tqw, tkw), EPS, tcs, rot)
    q = R.qk_norm_rope(tqkv, 0, 128, H, 128, tqw, EPS, True, tcs, rot)
    k = R.qk_norm_rope(tqkv, inner, 128, H, 128, tkw, EPS, True, tcs, rot)
    km = h3q.attn_kmean(k)
    q8, qs = R.quant_heads(q)
    k8, ks = R.quant_heads(k, km)
    v16 = R.v_to_f16(tqkv, 3 * inner, 2 * inner, S, H)
    ref = R.attn_qk8(q8, qs, k8, ks, v16, O.attn_scale_log2())
    err = O.max_abs_rel(out.float().cpu().numpy().reshape(S, H, 128), ref.float().cpu().numpy())
    assert err <= TOL, err


def test_attend_qkv_rejects_unsupported(cuda):
    S, H = 64, 1
    qkv = torch.zeros((S, 3 * 128), dtype=torch.bfloat16, device=cuda)
    cs = torch.zeros((2, S, 5), device=cuda)
    with pytest.raises(h3q.H3QError):
        h3q.attend_qkv(qkv, H, None, EPS, cs, 10)  # rot % 8 != 0
    with pytest.raises(h3q.H3QError):
        h3q.attend_qkv(qkv, H, None, EPS, None, 0, flags=8)
    with pytest.raises(h3q.H3QError, match="multiples of 8"):
        h3q.attend_qkv(torch.zeros((S, 3 * 128 + 4), dtype=torch.bfloat16, device=cuda), H, None, EPS, None, 0)
    x = torch.zeros((S, 600), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(h3q.H3QError):
        h3q.qk_norm_rope(x, 0, 1, 300)  # head_dim > 256
