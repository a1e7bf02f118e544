"""GPU parity of the tcgen05 int8 GEMM and its epilogues.

int32 accumulators and integer codes must be bit-exact; the bf16 outputs of the linear epilogue are computed
with the reference's exact multiply-add order and are checked bit-exact too; SwiGLU / GELU outputs (which call
__expf / tanhf on the device and expf / tanhf on the CPU) are checked within max-abs-rel 1e-2."""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_bits, bf16_tensor, linear_inputs, t

pytestmark = pytest.mark.gpu
TOL = 1e-2

ACC_SHAPES = [(1, 64, 16), (128, 256, 256), (129, 1024, 272), (300, 5120, 512), (257, 13824, 256),
              (64, 128, 1024), (1000, 2048, 48), (513, 5376, 784)]


@pytest.mark.parametrize("M,K,N", ACC_SHAPES)
def test_acc_int32_bit_exact(cuda, M, K, N):
    rng = np.random.default_rng(M + K + N)
    a = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    b = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    acc = h3q.gemm_s8_acc(t(a, cuda), t(b, cuda)).cpu().numpy()
    want = (a.astype(np.float64) @ b.astype(np.float64).T).astype(np.int64)
    assert np.array_equal(acc.astype(np.int64), want)


def test_acc_extreme_codes(cuda):
    """All -128 / 127 codes: the largest accumulators the int8 range allows."""
    M, K, N = 130, 13824, 256
    a = np.full((M, K), -128, dtype=np.int8)
    b = np.full((N, K), -128, dtype=np.int8)
    b[1::2] = 127
    acc = h3q.gemm_s8_acc(t(a, cuda), t(b, cuda)).cpu().numpy()
    assert np.all(acc[:, 0::2] == 128 * 128 * K) and np.all(acc[:, 1::2] == -128 * 127 * K)


@pytest.mark.parametrize("M,K,N", [(256, 1024, 1024), (77, 5120, 512), (129, 13824, 256), (1, 256, 16),
                                   (300, 2048, 384), (512, 1024, 640)])
@pytest.mark.parametrize("rotate", [True, False])
def test_gemm_s8_bit_exact_vs_oracle(cuda, M, K, N, rotate):
    (x, w, ws, bias), (xd, wd, wsd, bd) = linear_inputs(M + N, M, K, N, cuda)
    out = bf16_bits(h3q.gemm_s8(xd, wd, wsd, bd, swiglu=False, rotate=rotate))
    want, _, _, _ = O.gemm_s8(x, w, ws, bias, swiglu=False, rotate=rotate)
    assert np.array_equal(out, want)


def test_gemm_s8_scalar_scale_and_no_bias(cuda):
    (x, w, ws, _), (xd, wd, wsd, _) = linear_inputs(5, 200, 1024, 512, cuda)
    out = bf16_bits(h3q.gemm_s8(xd, wd, wsd[:1], None, rotate=True))
    q, xs = O.quant_rows(x, 2, O.QUANT_ROT2)
    want = O.gemm_s8_epilogue(O.gemm_s8_acc(q, w), xs, ws[:1], None)
    assert np.array_equal(out, want)


@pytest.mark.parametrize("rotate", [True, False])
def test_gemm_s8_swiglu_pairs(cuda, rotate):
    (x, w, ws, bias), (xd, wd, wsd, bd) = linear_inputs(21, 190, 2048, 768, cuda)
    out = bf16_bits(h3q.gemm_s8(xd, wd, wsd, bd, swiglu=True, rotate=rotate))
    want, _, _, _ = O.gemm_s8(x, w, ws, bias, swiglu=True, rotate=rotate)
    assert out.shape == (190, 384)
    assert O.max_abs_rel(O.bf16_bits_to_f32(out), O.bf16_bits_to_f32(want)) < TOL


@pytest.mark.parametrize("okind,dtype", [(0, torch.float32), (1, torch.float16), (2, torch.bfloat16)])
@pytest.mark.parametrize("swiglu", [False, True])
def test_int8_linear_ex_kinds(cuda, okind, dtype, swiglu):
    """kernels::int8_linear_ex: quant_rows_i8_rot codes, split-half SwiGLU, f32/f16/bf16 outputs."""
    M, K, N = 150, 1024, 512
    (x, w, ws, bias), (xd, wd, wsd, bd) = linear_inputs(okind + 10 * swiglu, M, K, N, cuda)
    out = h3q.int8_linear_ex(xd, wd, wsd, bd, dtype, swiglu=swiglu, rotate=True)
    q, xs = O.quant_rows(x, 2, O.QUANT_ROT)
    want = O.int8_epilogue(O.gemm_s8_acc(q, w), xs, ws, bias, okind, swiglu)
    got = out.cpu().numpy() if okind == 0 else out.view(torch.int16).cpu().numpy().view(np.uint16)
    if okind == 1:
        got_f, want_f = got.view(np.float16).astype(np.float32), want.view(np.float16).astype(np.float32)
    elif okind == 2:
        got_f, want_f = O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want)
    else:
        got_f, want_f = got, want
    if swiglu:
        assert O.max_abs_rel(got_f, want_f) < TOL
    else:
        assert np.array_equal(got_f, want_f)


def test_gelu_and_gate_resid_epilogues(cuda):
    M, K, N = 140, 1024, 768
    (x, w, ws, bias), (xd, wd, wsd, bd) = linear_inputs(33, M, K, N, cuda)
    q, xs = h3q.quant_rows(xd, True)
    qo, xso = O.quant_rows(x, 2, O.QUANT_ROT2)
    acc = O.gemm_s8_acc(qo, w)
    gelu = bf16_bits(h3q.gemm_s8_quantized(q, xs, wd, wsd, bd, h3q.EPI_GELU_TANH))
    want = O.gemm_s8_epilogue(acc, xso, ws, bias, O.EPI_GELU)
    assert O.max_abs_rel(O.bf16_bits_to_f32(gelu), O.bf16_bits_to_f32(want)) < TOL
    rng = np.random.default_rng(3)
    gate = O.bf16_round(rng.random((3, N), dtype=np.float32))
    idx = rng.integers(0, 3, size=M).astype(np.uint32)
    resid = O.f32_to_bf16_bits(rng.standard_normal((M, N)).astype(np.float32))
    gr = bf16_bits(h3q.gemm_s8_quantized(q, xs, wd, wsd, bd, h3q.EPI_GATE_RESID, gate=t(gate, cuda),
                                         gate_idx=t(idx, cuda), resid=bf16_tensor(resid, cuda)))
    want = O.gemm_s8_epilogue(acc, xso, ws, bias, O.EPI_GATE_RESID, gate=gate, gate_idx=idx, resid=resid)
    assert np.array_equal(gr, want)


def test_k_zero_gives_bias(cuda):
    a = torch.empty((5, 0), dtype=torch.int8, device=cuda)
    w = torch.empty((32, 0), dtype=torch.int8, device=cuda)
    xs = torch.ones(5, device=cuda)
    ws = torch.ones(32, device=cuda)
    bias = torch.arange(32, dtype=torch.float32, device=cuda)
    out = h3q.gemm_s8_quantized(a, xs, w, ws, bias, h3q.EPI_LINEAR, out_dtype=torch.float32)
    assert torch.equal(out, bias.expand(5, 32))


@pytest.mark.skipif(not R.available(), reason="reference comparator not built")
@pytest.mark.parametrize("swiglu", [False, True])
def test_gemm_matches_reference_gemm_s8_kernel(cuda, swiglu):
    """The reference's own gemm_s8 kernel on this GPU, fed the same codes, gives the same bf16 outputs."""
    M, K, N = 300, 5120, 1024
    (_, _, _, _), (xd, wd, wsd, bd) = linear_inputs(44, M, K, N, cuda)
    q, xs = h3q.quant_rows(xd, True)
    ref = R.gemm_s8(q, wd, xs, wsd, bd, swiglu)
    ours = h3q.gemm_s8_quantized(q, xs, wd, wsd, bd, h3q.EPI_SWIGLU_PAIRS if swiglu else h3q.EPI_LINEAR)
    torch.cuda.synchronize()
    assert torch.equal(ref.view(torch.int16), ours.view(torch.int16))


@pytest.mark.skipif(not R.available(), reason="reference comparator not built")
def test_split_swiglu_matches_reference_epilogue(cuda):
    M, K, N = 96, 1024, 512
    (_, _, _, _), (xd, wd, wsd, bd) = linear_inputs(45, M, K, N, cuda)
    q, xs = h3q.quant_rows(xd, True)
    acc = h3q.gemm_s8_acc(q, wd)
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        ref = R.int8_epilogue(acc, xs, wsd, bd, dt, True)
        ours = h3q.gemm_s8_quantized(q, xs, wd, wsd, bd, h3q.EPI_SWIGLU_HALVES, out_dtype=dt)
        assert torch.equal(ref, ours)


def test_full_size_c1_checksums(cuda):
    """M=32760, K=5120, N=13824: sampled rows bit-exact against the oracle, and row / column
    checksums of all int32 accumulators against exact CPU sums of the GPU's own codes."""
    M, K, N = 32760, 5120, 13824
    g = torch.Generator(device=cuda).manual_seed(1)
    xd = torch.randn((M, K), generator=g, device=cuda).to(torch.bfloat16)
    wd = torch.randint(-127, 128, (N, K), generator=g, device=cuda, dtype=torch.int8)
    wsd = torch.rand(N, generator=g, device=cuda) * 9e-3 + 1e-3
    bd = (torch.randn(N, generator=g, device=cuda) * 0.02).to(torch.bfloat16).float()
    out = h3q.gemm_s8(xd, wd, wsd, bd, swiglu=False, rotate=True)
    q, xs = h3q.quant_rows(xd, True)
    acc = h3q.gemm_s8_acc(q, wd)
    rows = np.r_[0:8, 16380:16388, M - 16:M]
    x_rows = bf16_bits(xd[rows])
    w = wd.cpu().numpy()
    qo, so = O.quant_rows(x_rows, 2, O.QUANT_ROT2)
    assert np.array_equal(q[rows].cpu().numpy(), qo)
    want = O.gemm_s8_epilogue(O.gemm_s8_acc(qo, w), so, wsd.cpu().numpy(), bd.cpu().numpy())
    assert np.array_equal(bf16_bits(out[rows]), want)
    qh = q.cpu().numpy().astype(np.float64)
    wf = w.astype(np.float64)
    col = acc.to(torch.float64).sum(0).cpu().numpy()
    assert np.array_equal(col, qh.sum(0) @ wf.T)
    row = acc.to(torch.float64).sum(1).cpu().numpy()
    assert np.array_equal(row, qh @ wf.sum(0))
