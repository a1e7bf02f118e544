"""GPU tests of checkpoint loading (h3q_checkpoint_upload, QLinear::load, weights.rs:493-534): the bytes that
reach the device through the pinned staging equal the file's, the (gate, up) interleave done by the copy equals
interleave_rows, and layers loaded from a file give the same outputs, bit for bit, as the same tensors handed to
the library directly.
"""
import pytest
import torch

import h3q
from h3q import checkpoint as C

pytestmark = pytest.mark.gpu

pytest.importorskip("safetensors")
from tests.test_checkpoint import PFX, make_checkpoint  # noqa: E402
from safetensors.torch import save_file  # noqa: E402


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    p = tmp_path_factory.mktemp("gpu_ckpt") / "model.safetensors"
    return p, make_checkpoint(p, seed=1)


def test_upload_equals_file(cuda, ckpt):
    path, tensors = ckpt
    with C.SafeFile(path) as f:
        for k, t in tensors.items():
            name = k[len(PFX):] if k.startswith(PFX) else k
            d = f.load(name, cuda)
            want = t.reshape(-1).contiguous().view(torch.uint8)
            assert torch.equal(d.reshape(-1).view(torch.uint8).cpu(), want), name


def test_large_and_interleaved_uploads(cuda, tmp_path):
    """Tensors larger than the 16 MiB staging chunk (several overlapped chunks), interleaved rows of both the
    whole-rows path and the split-row path (rows larger than a chunk)."""
    g = torch.Generator().manual_seed(5)
    t = {"big": torch.randint(-128, 128, (4096, 5120), generator=g, dtype=torch.int8),          # 20 MiB
         "wide": torch.randint(0, 256, (4, 20 << 20), generator=g, dtype=torch.uint8),          # 20 MiB rows
         "rows": torch.randint(-128, 128, (10, 7), generator=g, dtype=torch.int8)}
    p = tmp_path / "big.safetensors"
    save_file(t, str(p))
    with C.SafeFile(p) as f:
        assert torch.equal(f.load("big", cuda).cpu(), t["big"])
        for name in t:
            got = f.load(name, cuda, interleave=True).cpu()
            assert torch.equal(got, C.interleave_rows(t[name])), name
        assert torch.equal(f.load("wide", cuda).cpu(), t["wide"])


def test_int8_layer_from_file(cuda, ckpt):
    path, tensors = ckpt
    x = (torch.randn((300, 256), device=cuda) * 2).to(torch.bfloat16)
    with C.SafeFile(path) as f:
        for prefix in ("blocks.0.attn.qkv", "blocks.0.ff.fc2"):
            layer = C.load_qlinear(f, prefix, cuda)
            w = tensors[PFX + prefix + ".weight"].to(cuda)
            sc = tensors[PFX + prefix + ".weight_scale"].to(cuda)
            b = tensors.get(PFX + prefix + ".bias")
            direct = h3q.QLinear(w, sc, None if b is None else b.to(cuda), convrot=layer.desc.convrot)
            xin = x if layer.desc.in_features == 256 else torch.cat([x, x], dim=1)
            assert torch.equal(layer.forward(xin).view(torch.int16), direct.forward(xin).view(torch.int16)), prefix
    assert h3q.device_status() == 0


def test_swiglu_layer_interleaved_by_the_upload(cuda, ckpt):
    """interleave_swiglu applied while loading equals the interleave done on the device tensors, and the layer
    loaded without it runs the split-half SwiGLU path exactly as the same tensors handed over directly."""
    path, tensors = ckpt
    x = (torch.randn((200, 256), device=cuda) * 2).to(torch.bfloat16)
    with C.SafeFile(path) as f:
        il = C.load_qlinear(f, "blocks.0.ff.fc1", cuda, interleave_swiglu=True)
        plain = C.load_qlinear(f, "blocks.0.ff.fc1", cuda)
    w = tensors[PFX + "blocks.0.ff.fc1.weight"].to(cuda)
    sc = tensors[PFX + "blocks.0.ff.fc1.weight_scale"].to(cuda)
    b = tensors[PFX + "blocks.0.ff.fc1.bias"].to(cuda)
    direct = h3q.QLinear(C.interleave_rows(w).contiguous(), C.interleave_rows(sc).contiguous(),
                         C.interleave_rows(b).contiguous(), convrot=256, interleaved=True)
    y = il.run_swiglu(x)
    assert torch.equal(y.view(torch.int16), direct.run_swiglu(x).view(torch.int16))
    direct_plain = h3q.QLinear(w, sc, b, convrot=256)
    assert torch.equal(plain.run_swiglu(x).view(torch.int16), direct_plain.run_swiglu(x).view(torch.int16))
    assert h3q.device_status() == 0


def test_nvfp4_layer_from_file(cuda, ckpt):
    path, tensors = ckpt
    x = torch.randn((64, 256), device=cuda).to(torch.bfloat16)
    with C.SafeFile(path) as f:
        layer = C.load_qlinear(f, "text.mlp.up", cuda)
    assert (layer.out_features, layer.in_features) == (128, 256)
    q = tensors["text.mlp.up.weight"].to(cuda)
    bs = tensors["text.mlp.up.weight_scale"].view(torch.uint8).to(cuda)
    g = tensors["text.mlp.up.weight_scale_2"].reshape(1).to(cuda)
    pq = tensors["text.mlp.up.pre_quant_scale"].to(cuda)
    want = h3q.nvfp4_linear(x, q, bs, g, pq, None)
    assert torch.equal(layer.forward(x).view(torch.int16), want.view(torch.int16))
    assert h3q.device_status() == 0
