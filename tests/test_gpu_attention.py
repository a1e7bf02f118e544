"""GPU parity of the int8 attention (attn8.rs) against the CPU oracle and the reference's own kernels.

Bit-exact: the K column mean (fixed summation order), the int8 codes and scales of QuantHeads (per token and
per 128-token block), the V relayout, and the int32 Q.K^T accumulators of the tcgen05 kernel.  Within
tolerance (max|y - r| / max|r| <= 1e-2, the bf16 output contract): the attention output against the oracle's
restatement of attn_qk8 and against attn_qk8 itself compiled for sm_100a.
"""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_bits, bf16_tensor, t

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _inputs(seed, S, H, dev, k_offset=3.0):
    q, k, v = O.make_attn_inputs(seed, S, H, k_offset)
    return (q, k, v), (bf16_tensor(q, dev), bf16_tensor(k, dev), bf16_tensor(v, dev))


@pytest.mark.parametrize("S,H", [(1, 1), (37, 2), (300, 3), (1000, 2)])
def test_kmean_bit_exact(cuda, S, H):
    (q, k, v), (tq, tk, tv) = _inputs(11, S, H, cuda)
    got = h3q.attn_kmean(tk).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), O.attn_kmean(k).view(np.uint32))


@pytest.mark.parametrize("block", [False, True])
@pytest.mark.parametrize("S,H", [(1, 1), (129, 2), (300, 3), (777, 1)])
def test_quant_heads_bit_exact(cuda, S, H, block):
    (q, k, v), (tq, tk, tv) = _inputs(12, S, H, cuda)
    km = O.attn_kmean(k)
    flags = h3q.ATTN_SCALE_BLOCK128 if block else 0
    for x_np, x_t, mean in ((q, tq, None), (k, tk, km)):
        codes, scales = h3q.attn_quant_heads(x_t, None if mean is None else t(mean, cuda), flags)
        rc, rs = O.attn_quant_heads(x_np, mean, block)
        np.testing.assert_array_equal(codes.cpu().numpy(), rc)
        np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_quant_heads_edge_values(cuda):
    """Rows of zeros (scale floor 1e-20), NaN and +-inf elements, huge values: codes and scales as the oracle."""
    S, H = 64, 2
    x = np.zeros((S, H, 128), dtype=np.float32)
    x[1, 0, :] = 1e30
    x[2, 1, 5] = np.nan
    x[3, 0, 7] = np.inf
    x[4, 1, 9] = -np.inf
    x[5, 0, :] = np.linspace(-3, 3, 128)
    x[6, 1, :] = 1e-30
    xb = O.f32_to_bf16_bits(x)
    for block in (False, True):
        codes, scales = h3q.attn_quant_heads(bf16_tensor(xb, cuda), None, h3q.ATTN_SCALE_BLOCK128 if block else 0)
        rc, rs = O.attn_quant_heads(xb, None, block)
        np.testing.assert_array_equal(codes.cpu().numpy(), rc)
        np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), rs.view(np.uint32))


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("S,H", [(200, 2), (1000, 3)])
def test_quant_heads_matches_reference_kernel(cuda, S, H):
    """The reference's QuantHeads kernel, given the same mean, yields the same codes and scales."""
    (q, k, v), (tq, tk, tv) = _inputs(13, S, H, cuda)
    km = h3q.attn_kmean(tk)
    for x_t, mean in ((tq, None), (tk, km)):
        codes, scales = h3q.attn_quant_heads(x_t, mean)
        rc, rs = R.quant_heads(x_t, mean)
        assert torch.equal(codes, rc)
        assert torch.equal(scales[:, :S].contiguous().view(torch.int32), rs.view(torch.int32))


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
def test_kmean_close_to_reference_kernel(cuda):
    """The reference sums its row chunks with atomicAdd (any order); the fixed order agrees to rounding."""
    (q, k, v), (tq, tk, tv) = _inputs(14, 4096, 3, cuda)
    got = h3q.attn_kmean(tk)
    ref = R.col_mean(tk)
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("S,H,rs,col", [(300, 2, 256, 0), (129, 3, 3 * 384, 768), (77, 2, 600, 6)])
def test_v_layout(cuda, S, H, rs, col, bf16):
    g = np.random.default_rng(5)
    src = O.f32_to_bf16_bits(g.standard_normal((S, rs)).astype(np.float32))
    flags = h3q.ATTN_PV_BF16 if bf16 else 0
    vt = h3q.attn_v_layout(bf16_tensor(src, cuda), rs, col, S, H, flags)
    Sp = (S + 127) // 128 * 128
    assert vt.shape == (H, 128, Sp)
    v = torch.from_numpy(O.bf16_bits_to_f32(src[:, col:col + H * 128]).reshape(S, H, 128))
    want = v.to(torch.bfloat16 if bf16 else torch.float16).permute(1, 2, 0)
    got = vt[:, :, :S].cpu()
    assert torch.equal(got.view(torch.int16), want.contiguous().view(torch.int16))


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
def test_v_layout_matches_reference_kernel(cuda):
    S, H = 300, 2
    g = np.random.default_rng(6)
    src = bf16_tensor(O.f32_to_bf16_bits(g.standard_normal((S, 3 * H * 128)).astype(np.float32)), cuda)
    vt = h3q.attn_v_layout(src, 3 * H * 128, 2 * H * 128, S, H)
    ref = R.v_to_f16(src, 3 * H * 128, 2 * H * 128, S, H)
    assert torch.equal(vt[:, :, :S].permute(0, 2, 1).contiguous().view(torch.int16), ref.view(torch.int16))


def _stages(q, k, v, dev, flags=0):
    S, H = q.shape[0], q.shape[1]
    block = bool(flags & h3q.ATTN_SCALE_BLOCK128)
    km = O.attn_kmean(k)
    q8, qs = O.attn_quant_heads(q, None, block)
    k8, ks = O.attn_quant_heads(k, km, block)
    vt = h3q.attn_v_layout(bf16_tensor(v, dev).reshape(S, H * 128), H * 128, 0, S, H, flags)
    return (q8, qs, k8, ks), (t(q8, dev), t(qs, dev), t(k8, dev), t(ks, dev), vt)


@pytest.mark.parametrize("S,H", [(1, 1), (100, 1), (256, 2), (300, 2), (640, 1)])
def test_scores_bit_exact(cuda, S, H):
    """The int32 Q.K^T accumulators of the tcgen05 kernel equal the integer dot products."""
    (q, k, v), _ = _inputs(21, S, H, cuda)
    (q8, qs, k8, ks), dev_stages = _stages(q, k, v, cuda)
    out, sc = h3q.attention_core(*dev_stages, scores=True)
    np.testing.assert_array_equal(sc.cpu().numpy(), O.attn_scores(q8, k8))
    assert h3q.device_status() == 0


@pytest.mark.parametrize("flags", [0, 1, 2, 3])
@pytest.mark.parametrize("S,H", [(1, 1), (129, 2), (300, 2), (1000, 1)])
def test_attention_core_vs_oracle(cuda, S, H, flags):
    (q, k, v), _ = _inputs(22, S, H, cuda)
    (q8, qs, k8, ks), dev_stages = _stages(q, k, v, cuda, flags)
    out = h3q.attention_core(*dev_stages, flags=flags)
    ref = O.attn_forward(q8, qs, k8, ks, v.reshape(S, H * 128), H * 128, 0, bool(flags & h3q.ATTN_PV_BF16))
    err = O.max_abs_rel(O.bf16_bits_to_f32(bf16_bits(out)), O.bf16_bits_to_f32(ref))
    assert err <= TOL, err
    assert h3q.device_status() == 0


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("S,H", [(300, 2), (2048, 2)])
def test_attention_core_vs_reference_kernel(cuda, S, H):
    """attn_qk8 itself (compiled for sm_100a) on the same codes, scales and V."""
    (q, k, v), (tq, tk, tv) = _inputs(23, S, H, cuda)
    km = h3q.attn_kmean(tk)
    q8, qs = h3q.attn_quant_heads(tq)
    k8, ks = h3q.attn_quant_heads(tk, km)
    vt = h3q.attn_v_layout(tv.reshape(S, H * 128), H * 128, 0, S, H)
    out = h3q.attention_core(q8, qs, k8, ks, vt)
    v16 = R.v_to_f16(tv.reshape(S, H * 128), H * 128, 0, S, H)
    ref = R.attn_qk8(q8, qs[:, :S].contiguous(), k8, ks[:, :S].contiguous(), v16, O.attn_scale_log2())
    err = O.max_abs_rel(out.float().cpu().numpy(), ref.float().cpu().numpy())
    assert err <= TOL, err
    # the oracle against the reference kernel: pins the oracle's restatement on the reference's device results
    oref = O.attn_forward(q8.cpu().numpy(), qs.cpu().numpy(), k8.cpu().numpy(), ks.cpu().numpy(),
                          v.reshape(S, H * 128), H * 128, 0)
    assert O.max_abs_rel(O.bf16_bits_to_f32(oref), ref.float().cpu().numpy()) <= TOL


@pytest.mark.parametrize("flags", [0, 3])
@pytest.mark.parametrize("S,H", [(300, 2), (1500, 1)])
def test_attention_pipeline(cuda, S, H, flags):
    """h3q.attention (attn8::attention) end to end against the oracle pipeline, and attention_qkv with V read
    out of a fused qkv activation gives the same bits."""
    (q, k, v), (tq, tk, tv) = _inputs(24, S, H, cuda)
    out = h3q.attention(tq, tk, tv, flags)
    ref = O.attention(q, k, v, flags)
    err = O.max_abs_rel(O.bf16_bits_to_f32(bf16_bits(out)), O.bf16_bits_to_f32(ref))
    assert err <= TOL, err
    qkv = torch.cat([tq.reshape(S, -1), tk.reshape(S, -1), tv.reshape(S, -1)], dim=1).contiguous()
    out2 = h3q.attention_qkv(tq, tk, qkv, 2 * H * 128, flags)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    # close to exact softmax attention (the int8 approximation itself)
    ex = O.attention_exact(q, k, v)
    assert O.max_abs_rel(O.bf16_bits_to_f32(bf16_bits(out)), ex) <= 5e-2
    assert h3q.device_status() == 0


def test_attention_rejects_bad_arguments(cuda):
    S, H = 64, 1
    x = torch.zeros((S, H, 128), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(h3q.H3QError):
        h3q.attention(x, x, x, flags=8)
    qkv = torch.zeros((S, 3 * 128), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(h3q.H3QError):
        h3q.attention_qkv(x, x, qkv, 3 * 128 - 64)


@pytest.mark.parametrize("lo,hi", [(0, 300), (100, 357), (513, 1000), (999, 1000)])
def test_attention_rows_equal_whole_sequence_rows(cuda, lo, hi):
    """A block of query rows against all keys gives exactly those rows of the whole-sequence attention, and the
    oracle's restatement of it."""
    S, H = 1000, 2
    (q, k, v), (tq, tk, tv) = _inputs(25, S, H, cuda)
    full = h3q.attention(tq, tk, tv)
    part = h3q.attention_rows(tq[lo:hi].contiguous(), tk, tv.reshape(S, H * 128), H * 128, 0)
    assert torch.equal(part.view(torch.int16), full[lo:hi].view(torch.int16))
    ref = O.attention_rows(q[lo:hi], k, v)
    assert O.max_abs_rel(O.bf16_bits_to_f32(bf16_bits(part)), O.bf16_bits_to_f32(ref)) <= TOL
