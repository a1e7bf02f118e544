"""CPU tests of the native checkpoint reader (h3q_checkpoint_*, the reference's SafeFile and QLinear::load,
weights.rs:23-139 and :493-534).

Fixtures are written with the safetensors package itself, so the reader is checked against the format's own
writer: names (with the ComfyUI prefix stripped), dtypes, shapes, bytes, metadata, the `comfy_quant` records of
int8_tensorwise (+ ConvRot), nvfp4 and dense layers, the SwiGLU row interleave, and the errors for broken files.
"""
import json
import os
import struct

import numpy as np
import pytest
import torch

import h3q
from h3q import checkpoint as C

safetensors = pytest.importorskip("safetensors")
from safetensors import safe_open  # noqa: E402
from safetensors.torch import save_file  # noqa: E402

PFX = "model.diffusion_model."


def _quant(conf: dict) -> torch.Tensor:
    return torch.tensor(list(json.dumps(conf).encode()), dtype=torch.uint8)


def make_checkpoint(path, seed=0):
    g = torch.Generator().manual_seed(seed)
    t = {
        # int8 + ConvRot layer with per-row scale and bias (the DiT's linears)
        PFX + "blocks.0.attn.qkv.weight": torch.randint(-127, 128, (512, 256), generator=g, dtype=torch.int8),
        PFX + "blocks.0.attn.qkv.weight_scale": torch.rand(512, generator=g) * 1e-2,
        PFX + "blocks.0.attn.qkv.bias": (torch.randn(512, generator=g) * 0.02).to(torch.bfloat16),
        PFX + "blocks.0.attn.qkv.comfy_quant": _quant({"format": "int8_tensorwise", "convrot": True,
                                                       "convrot_groupsize": 256}),
        # int8 with a scalar scale, no rotation, no bias
        PFX + "blocks.0.ff.fc2.weight": torch.randint(-127, 128, (256, 512), generator=g, dtype=torch.int8),
        PFX + "blocks.0.ff.fc2.weight_scale": torch.tensor(3e-3),
        PFX + "blocks.0.ff.fc2.comfy_quant": _quant({"format": "int8_tensorwise"}),
        # gate/up projection (SwiGLU) with per-row scale and f32 bias, default group size
        PFX + "blocks.0.ff.fc1.weight": torch.randint(-127, 128, (1024, 256), generator=g, dtype=torch.int8),
        PFX + "blocks.0.ff.fc1.weight_scale": torch.rand(1024, generator=g) * 1e-2,
        PFX + "blocks.0.ff.fc1.bias": torch.randn(1024, generator=g) * 0.02,
        PFX + "blocks.0.ff.fc1.comfy_quant": _quant({"format": "int8_tensorwise", "convrot": True}),
        # an NVFP4 text-encoder layer: packed e2m1, e4m3 block scales (128x4 swizzle: 128 rows x 4 atoms), global
        "text.mlp.up.weight": torch.randint(0, 256, (128, 128), generator=g, dtype=torch.uint8),
        "text.mlp.up.weight_scale": (torch.rand((128, 16), generator=g) + 0.5).to(torch.float8_e4m3fn),
        "text.mlp.up.weight_scale_2": torch.tensor(0.01),
        "text.mlp.up.pre_quant_scale": (1 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16),
        "text.mlp.up.comfy_quant": _quant({"format": "nvfp4"}),
        # a dense layer and an unknown format
        "norm.proj.weight": torch.randn((64, 128), generator=g).to(torch.bfloat16),
        "bad.layer.weight": torch.zeros((8, 8), dtype=torch.int8),
        "bad.layer.comfy_quant": _quant({"format": "int4_magic"}),
        # other storage dtypes
        "misc.f16": torch.randn(5, generator=g).to(torch.float16),
        "misc.i64": torch.arange(7, dtype=torch.int64),
        "misc.f64": torch.randn((2, 3), generator=g, dtype=torch.float64),
        "misc.bool": torch.tensor([True, False, True]),
        "misc.empty": torch.zeros((0, 4), dtype=torch.float32),
    }
    save_file(t, str(path), metadata={"format": "pt", "modelspec.title": "h3 test é"})
    return t


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    p = tmp_path_factory.mktemp("ckpt") / "model.safetensors"
    return p, make_checkpoint(p)


def test_names_info_and_bytes_match_the_format_writer(ckpt):
    path, tensors = ckpt
    with C.SafeFile(path) as f, safe_open(str(path), framework="pt") as ref:
        want = sorted(k[len(PFX):] if k.startswith(PFX) else k for k in tensors)
        assert f.names() == want
        for k in ref.keys():
            name = k[len(PFX):] if k.startswith(PFX) else k
            assert f.has(name)
            dt, shape, nbytes = f.info(name)
            sl = ref.get_slice(k)
            assert dt == sl.get_dtype()
            assert list(shape) == list(sl.get_shape())
            t = ref.get_tensor(k)
            assert nbytes == t.numel() * t.element_size()
            raw = t.reshape(-1).contiguous().view(torch.uint8).numpy().tobytes()
            assert f.read(name).tobytes() == raw
            cpu = f.load(name, "cpu")
            assert cpu.dtype == (torch.uint8 if t.dtype in (torch.float8_e4m3fn, torch.bool) else t.dtype)
            assert cpu.reshape(-1).view(torch.uint8).numpy().tobytes() == raw
        assert not f.has("blocks.0.attn.qkv.missing")
        assert not f.has(PFX + "blocks.0.attn.qkv.weight")  # stored with the prefix, found without it


def test_metadata(ckpt):
    path, _ = ckpt
    with C.SafeFile(path) as f:
        assert f.metadata("format") == "pt"
        assert f.metadata("modelspec.title") == "h3 test é"
        assert f.metadata("nope") is None


def test_qlinear_specs(ckpt):
    path, _ = ckpt
    with C.SafeFile(path) as f:
        s = f.qlinear_spec("blocks.0.attn.qkv")
        assert (s.format, s.convrot, s.out_features, s.in_features) == (h3q.FMT_INT8, 256, 512, 256)
        assert (s.scale_numel, s.has_bias, s.weight_dtype) == (512, 1, C.DT_I8)
        s = f.qlinear_spec("blocks.0.ff.fc2")
        assert (s.format, s.convrot, s.scale_numel, s.has_bias) == (h3q.FMT_INT8, 0, 1, 0)
        s = f.qlinear_spec("blocks.0.ff.fc1")
        assert (s.convrot, s.out_features) == (256, 1024)  # "convrot": true without a group size -> 256
        s = f.qlinear_spec("text.mlp.up")
        assert (s.format, s.out_features, s.in_features) == (h3q.FMT_NVFP4, 128, 256)
        assert (s.has_pre_quant_scale, s.scale_dtype, s.scale_numel) == (1, C.DT_F8_E4M3, 128 * 16)
        s = f.qlinear_spec("norm.proj")
        assert (s.format, s.in_features) == (h3q.FMT_DENSE, 128)
        assert f.comfy_quant("blocks.0.attn.qkv") == {"format": "int8_tensorwise", "convrot": True,
                                                      "convrot_groupsize": 256}
        assert f.comfy_quant("norm.proj") is None
        with pytest.raises(h3q.H3QError, match="unsupported quantization format int4_magic"):
            f.qlinear_spec("bad.layer")
        with pytest.raises(h3q.H3QError, match="tensor nope.weight not found"):
            f.qlinear_spec("nope")


def test_host_interleave(ckpt):
    path, tensors = ckpt
    with C.SafeFile(path) as f:
        w = f.load("blocks.0.ff.fc1.weight", "cpu", interleave=True)
        ref = tensors[PFX + "blocks.0.ff.fc1.weight"]
        assert torch.equal(w[0::2], ref[:512]) and torch.equal(w[1::2], ref[512:])
        layer = C.load_qlinear(f, "blocks.0.ff.fc1", "cpu", interleave_swiglu=True)
        assert layer.desc.interleaved == 1 and layer.desc.convrot == 256
        b = tensors[PFX + "blocks.0.ff.fc1.bias"]
        assert torch.equal(layer.bias[0::2], b[:512]) and torch.equal(layer.bias[1::2], b[512:])
        sc = tensors[PFX + "blocks.0.ff.fc1.weight_scale"]
        assert torch.equal(layer.scale[0::2], sc[:512]) and torch.equal(layer.scale[1::2], sc[512:])


def _raw_file(path, header, data=b""):
    hb = header if isinstance(header, bytes) else json.dumps(header).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(hb)) + hb + data)


def test_header_json_details(tmp_path):
    """Escapes and unicode in names, padding spaces, non-string metadata (kept as its JSON text)."""
    p = tmp_path / "esc.safetensors"
    hdr = ('{"__metadata__": {"n": 3, "s": "x\\ty", "o": {"a": [1, true, null]}}, '
           '"na\\"me\\u00e9\\ud83d\\ude00": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}    ').encode()
    _raw_file(p, hdr, struct.pack("<2f", 1.5, -2.0))
    with C.SafeFile(p) as f:
        assert f.names() == ['na"meé\U0001F600']
        np.testing.assert_array_equal(f.read('na"meé\U0001F600'), [1.5, -2.0])
        assert f.metadata("n") == "3"
        assert f.metadata("s") == "x\ty"
        assert f.metadata("o") == '{"a":[1,true,null]}'


@pytest.mark.parametrize("case,msg", [
    ("short", "not a safetensors file"),
    ("hdrlen", "does not fit the file"),
    ("json", "bad header JSON"),
    ("offsets", "outside the"),
    ("size", "bytes for a BF16 tensor"),
    ("dtype", "unsupported safetensors dtype"),
    ("shape", "malformed entry"),
])
def test_broken_files_are_rejected(tmp_path, case, msg):
    p = tmp_path / f"{case}.safetensors"
    ok = {"t": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]}}
    if case == "short":
        p.write_bytes(b"\x01\x02")
    elif case == "hdrlen":
        p.write_bytes(struct.pack("<Q", 1 << 20) + b"{}")
    elif case == "json":
        _raw_file(p, b'{"t": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]', b"\0" * 8)
    elif case == "offsets":
        _raw_file(p, {"t": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 16]}}, b"\0" * 8)
    elif case == "size":
        _raw_file(p, {"t": {"dtype": "BF16", "shape": [2, 3], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "dtype":
        _raw_file(p, {"t": {"dtype": "F4", "shape": [2, 2], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "shape":
        _raw_file(p, {"t": {"dtype": "BF16", "shape": "2x2", "data_offsets": [0, 8]}}, b"\0" * 8)
    with pytest.raises(h3q.H3QError, match=msg):
        C.SafeFile(p)
    _raw_file(tmp_path / "fine.safetensors", ok, b"\0" * 8)
    with C.SafeFile(tmp_path / "fine.safetensors") as f:
        assert f.info("t") == ("BF16", (2, 2), 8)


def test_missing_file_and_tensor(tmp_path, ckpt):
    with pytest.raises(h3q.H3QError, match="opening"):
        C.SafeFile(tmp_path / "absent.safetensors")
    with C.SafeFile(ckpt[0]) as f:
        with pytest.raises(h3q.H3QError, match="not found"):
            f.read("nope")
        with pytest.raises(ValueError):
            C.interleave_rows(np.zeros((3, 2)))
