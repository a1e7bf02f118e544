"""CPU tests of the LoRA merge (QLinear::merge_loras, weights.rs:692-761) in the oracle, and of the LoRA file
reader (lora.rs:11-72) and the merge driver's host logic (dit.rs:654-690).

The reference forms its f32 matmuls (b @ a and the rotations) in an order the BLAS picks, so no golden vector pins
the merged codes; the oracle's fixed-order f32 restatement is checked here against an order-free f64 restatement
(exact rotation, no rounding before the codes): codes within one step, nearly all identical.  The zero-delta case
is a known answer: merging a zero delta into rows whose largest code is +-127 returns the same codes.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

RNG_SEED = 7


def _bf16(x):
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def make_layer(n, k, seed, per_row=True, full_range=True):
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, (n, k)).astype(np.int8)
    if full_range:  # every row reaches +-127, so the zero-delta merge is the identity on codes
        q[np.arange(n), rng.integers(0, k, n)] = 127
    s = rng.uniform(1e-3, 1e-2, n if per_row else 1).astype(np.float32)
    return q, s


def make_loras(n, k, ranks, seed, scales=None):
    rng = np.random.default_rng(seed)
    out = []
    for i, r in enumerate(ranks):
        a = _bf16(rng.standard_normal((r, k)) * 0.05)
        b = _bf16(rng.standard_normal((n, r)) * 0.05)
        out.append((a, b, (scales or [0.75] * len(ranks))[i]))
    return out


@pytest.mark.parametrize("convrot,per_row,ranks", [(256, True, [16]), (256, True, [8, 3]), (0, True, [4]),
                                                   (256, False, [12]), (0, False, [1, 2, 3])])
def test_oracle_matches_f64_restatement(convrot, per_row, ranks):
    n, k = 64, 768
    q, s = make_layer(n, k, RNG_SEED, per_row)
    loras = make_loras(n, k, ranks, RNG_SEED + 1)
    qo, so = O.lora_merge_i8(q, s, loras, convrot)
    qe, se = O.lora_merge_i8_f64(q, s, loras, convrot)
    d = np.abs(qo.astype(np.int32) - qe.astype(np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() < 1e-3
    assert np.abs(so.astype(np.float64) / se - 1).max() < 1e-6
    assert so.shape == (n,)


@pytest.mark.parametrize("convrot", [256, 0])
def test_zero_delta_keeps_codes(convrot):
    n, k = 48, 512
    q, s = make_layer(n, k, 3)
    loras = [(a, b * 0, sc) for a, b, sc in make_loras(n, k, [8], 4)]
    qo, so = O.lora_merge_i8(q, s, loras, convrot)
    assert np.array_equal(qo, q)
    assert np.abs(so / s - 1).max() < 4e-7


def test_no_lora_returns_inputs():
    q, s = make_layer(8, 256, 1)
    qo, so = O.lora_merge_i8(q, s, [], 256)
    assert qo is q or np.array_equal(qo, q)
    assert np.array_equal(so, s)


def test_scale_is_affine_multiply_and_codes_round_half_away():
    """One row, one column group, no rotation: w = q * s + delta, s' = max|w| * f32(1/127), codes
    round(w / s') with halves away from zero."""
    k = 256
    q = np.zeros((1, k), dtype=np.int8)
    s = np.array([1.0], dtype=np.float32)
    a = np.zeros((1, k), dtype=np.float32)
    a[0, 0], a[0, 1], a[0, 2] = 127.0, 0.5, -0.5    # w = 127, 0.5, -0.5 (s' = 127 * f32(1/127))
    b = np.ones((1, 1), dtype=np.float32)
    qo, so = O.lora_merge_i8(q, s, [(a, b, 1.0)], 0)
    want_s = np.float32(np.float32(127.0) * np.float32(1.0 / 127.0))
    assert so[0] == max(want_s, np.float32(1e-30))
    r = np.float32(0.5) / so[0]
    assert qo[0, 0] == 127
    assert qo[0, 1] == int(np.sign(r) * np.floor(abs(r) + 0.5))
    assert qo[0, 2] == -qo[0, 1]


def test_dense_merge_matches_f64():
    n, k = 32, 320
    rng = np.random.default_rng(11)
    w = rng.standard_normal((n, k)).astype(np.float32)
    loras = make_loras(n, k, [6, 2], 12, scales=[0.5, -1.25])
    out = O.lora_merge_dense(w, loras)
    want = w.astype(np.float64)
    for a, b, sc in loras:
        want = want + float(np.float32(sc)) * (b.astype(np.float64) @ a.astype(np.float64))
    assert np.abs(out - want).max() <= 1e-5 * np.abs(want).max()


# ------------------------------------------------------------------------------------------------ LoRA files

safetensors = pytest.importorskip("safetensors")
from safetensors.torch import save_file  # noqa: E402

from h3q import checkpoint as C  # noqa: E402


def write_lora(path, n, k, r, seed=0, style="AB", prefix="diffusion_model.", alpha=None, reshape=None,
               module="blocks.0.attn.qkv_proj", dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn((r, k), generator=g) * 0.05).to(dtype)
    b = (torch.randn((n, r), generator=g) * 0.05).to(dtype)
    up, down = ("lora_B", "lora_A") if style == "AB" else ("lora_up", "lora_down")
    t = {f"{prefix}{module}.{up}.weight": b, f"{prefix}{module}.{down}.weight": a}
    if alpha is not None:
        t[f"{prefix}{module}.alpha"] = torch.tensor(alpha, dtype=torch.bfloat16)
    if reshape is not None:
        t[f"{prefix}{module}.reshape_weight"] = torch.tensor(reshape, dtype=torch.int64)
    save_file(t, str(path))
    return a, b


@pytest.mark.parametrize("style,prefix,alpha", [("AB", "diffusion_model.", 8.0), ("updown", "", None),
                                                 ("updown", "diffusion_model.", 3.0)])
def test_lora_file_delta(tmp_path, style, prefix, alpha):
    p = tmp_path / "l.safetensors"
    a, b = write_lora(p, 96, 64, 4, style=style, prefix=prefix, alpha=alpha)
    with C.LoraFile(str(p)) as f:
        assert f.prefix == prefix
        d = f.delta("blocks.0.attn.qkv_proj", "cpu")
        assert f.delta("blocks.0.attn.out_proj", "cpu") is None
    assert d.a.dtype == torch.bfloat16 and d.b.dtype == torch.bfloat16
    assert torch.equal(d.a, a.to(torch.bfloat16)) and torch.equal(d.b, b.to(torch.bfloat16))
    want = 1.0 if alpha is None else float(torch.tensor(alpha, dtype=torch.bfloat16).float()) / 4.0
    assert d.scale == want
    assert d.reshape is None


def test_lora_file_conv_factors_flatten(tmp_path):
    """Factors stored with trailing 1x1 dims (conv-style) flatten from dimension 1 (lora.rs:54-55)."""
    p = tmp_path / "c.safetensors"
    g = torch.Generator().manual_seed(2)
    a = torch.randn((4, 64, 1, 1), generator=g)
    b = torch.randn((32, 4, 1, 1), generator=g)
    save_file({"m.lora_A.weight": a, "m.lora_B.weight": b}, str(p))
    with C.LoraFile(str(p)) as f:
        d = f.delta("m", "cpu")
    assert tuple(d.a.shape) == (4, 64) and tuple(d.b.shape) == (32, 4)


def test_apply_lora_skips_mismatched_and_reshaped(tmp_path):
    """dit.rs:657-661: a pair whose shapes do not fit the layer, or with reshape_weight, is skipped (no device
    work on this path)."""
    p = tmp_path / "s.safetensors"
    write_lora(p, 96, 64, 4, module="a")
    with C.LoraFile(str(p)) as f:
        layer = C.DenseLinear(torch.zeros((80, 64), dtype=torch.bfloat16))   # out_features 80 != 96
        merged, skipped = C.apply_lora({"a": layer, "missing": layer}, f, 1.0, "cpu")
    assert merged == [] and skipped == ["a"]
    p2 = tmp_path / "r.safetensors"
    write_lora(p2, 96, 64, 4, module="a", reshape=[128, 64])
    with C.LoraFile(str(p2)) as f:
        d = f.delta("a", "cpu")
        assert d.reshape == [128, 64]
        layer = C.DenseLinear(torch.zeros((96, 64), dtype=torch.bfloat16))
        merged, skipped = C.apply_lora({"a": layer}, f, 1.0, "cpu")
    assert merged == [] and skipped == ["a"]
