"""GPU tests of the LoRA merge (h3q_lora_merge_i8 / h3q_lora_merge_dense, QLinear::merge_loras,
weights.rs:692-761): codes and scales bit-identical to the oracle's fixed-order restatement for ConvRot and plain
layers, per-row and scalar scales, bf16 / f16 / f32 factors, ranks across the staging chunk, ragged rows and
columns, chunked workspaces and in-place merges; dense weights bit-identical after the cast; the argument checks;
and a merged layer loaded from files running through the int8 GEMM exactly as the oracle's merged codes do.
"""
import ctypes

import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from tests.test_oracle_lora import make_layer, make_loras

pytestmark = pytest.mark.gpu


def _dev_loras(loras, dev, dtype=torch.bfloat16):
    return [(torch.from_numpy(a).to(dtype).to(dev), torch.from_numpy(b).to(dtype).to(dev), s) for a, b, s in loras]


def _np_loras(dloras):
    return [(a.float().cpu().numpy(), b.float().cpu().numpy(), s) for a, b, s in dloras]


@pytest.mark.parametrize("n,k,convrot,per_row,ranks", [
    (300, 1024, 256, True, [16]),
    (64, 512, 256, True, [40, 5]),        # rank across two staging chunks, two deltas
    (97, 256, 256, False, [7]),            # scalar scale, ragged rows
    (130, 320, 0, True, [3]),              # plain, columns not a multiple of 256
    (33, 100, 0, False, [9, 1]),           # plain, k % 16 != 0 (unaligned rows), scalar scale
    (40, 512, 256, True, [0, 6]),          # a rank-0 delta
])
def test_merge_i8_bit_exact(cuda, n, k, convrot, per_row, ranks):
    q, s = make_layer(n, k, n + k, per_row)
    dl = _dev_loras(make_loras(n, k, ranks, n + 1, scales=[0.5, -1.5][:len(ranks)]), cuda)
    wq, ws = h3q.lora_merge_i8(torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda), dl, convrot=convrot)
    torch.cuda.synchronize()
    qo, so = O.lora_merge_i8(q, s, _np_loras(dl), convrot)
    assert np.array_equal(wq.cpu().numpy(), qo)
    assert np.array_equal(ws.cpu().numpy().view(np.uint32), so.view(np.uint32))
    assert h3q.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_merge_i8_factor_dtypes(cuda, dtype):
    n, k = 128, 512
    q, s = make_layer(n, k, 5)
    dl = _dev_loras(make_loras(n, k, [12], 6), cuda, dtype)
    wq, ws = h3q.lora_merge_i8(torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda), dl)
    qo, so = O.lora_merge_i8(q, s, _np_loras(dl), 256)
    assert np.array_equal(wq.cpu().numpy(), qo)
    assert np.array_equal(ws.cpu().numpy(), so)


def test_merge_i8_chunked_workspace_and_in_place(cuda):
    n, k = 200, 768
    q, s = make_layer(n, k, 9)
    dl = _dev_loras(make_loras(n, k, [8], 10), cuda)
    descs, keep = h3q._lora_descs(dl, n, k, cuda)
    L = h3q.lib()
    w = torch.from_numpy(q).to(cuda)
    sc = torch.from_numpy(s).to(cuda)
    one_pass_q, one_pass_s = h3q.lora_merge_i8(w, sc, dl)
    for rows in (64, 33, 1):   # workspaces for 64, 33 (rounded to 32) and 1 row(s)
        ws_bytes = 256 + rows * k * 4
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
        wi, si = w.clone(), sc.clone()   # in place
        h3q.check(L.h3q_lora_merge_i8(wi.data_ptr(), si.data_ptr(), n, 256, descs, 1, wi.data_ptr(), si.data_ptr(),
                                      n, k, ws.data_ptr(), ws_bytes, h3q._stream(cuda)))
        assert torch.equal(wi, one_pass_q) and torch.equal(si, one_pass_s), rows
    ws = torch.empty(256 + k * 4 - 4, dtype=torch.uint8, device=cuda)
    with pytest.raises(h3q.H3QError, match="workspace"):
        h3q.check(L.h3q_lora_merge_i8(w.data_ptr(), sc.data_ptr(), n, 256, descs, 1, w.data_ptr(), sc.data_ptr(),
                                      n, k, ws.data_ptr(), ws.numel(), h3q._stream(cuda)))
    del keep


def test_zero_delta_keeps_codes(cuda):
    n, k = 256, 1024
    q, s = make_layer(n, k, 21)
    dl = [(a, b * 0, sc) for a, b, sc in _dev_loras(make_loras(n, k, [8], 22), cuda)]
    wq, _ = h3q.lora_merge_i8(torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda), dl)
    assert np.array_equal(wq.cpu().numpy(), q)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_merge_dense_bit_exact(cuda, dtype):
    n, k = 150, 384
    g = torch.Generator().manual_seed(3)
    w = torch.randn((n, k), generator=g).to(dtype)
    dl = _dev_loras(make_loras(n, k, [10, 4], 31, scales=[0.25, 2.0]), cuda)
    out = h3q.lora_merge_dense(w.to(cuda), dl)
    ref = O.lora_merge_dense(w.float().numpy(), _np_loras(dl))
    want = torch.from_numpy(ref).to(dtype)   # torch's f32 -> dtype casts round to nearest even, as candle's
    assert torch.equal(out.cpu().view(torch.uint8), want.view(torch.uint8))
    w_in = w.to(cuda)
    h3q.lora_merge_dense(w_in, dl, out=w_in)   # in place
    assert torch.equal(w_in.cpu().view(torch.uint8), want.view(torch.uint8))


def test_merge_argument_checks(cuda):
    n, k = 64, 512
    q, s = make_layer(n, k, 1, per_row=False)
    w, sc = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    dl = _dev_loras(make_loras(n, k, [4], 2), cuda)
    descs, keep = h3q._lora_descs(dl, n, k, cuda)
    L = h3q.lib()
    ws = torch.empty(h3q.lib().h3q_lora_merge_i8_workspace_size(n, k), dtype=torch.uint8, device=cuda)
    st = h3q._stream(cuda)
    out = torch.empty_like(w)
    out_s = torch.empty(n, dtype=torch.float32, device=cuda)
    args = lambda **kw: dict(dict(w=w.data_ptr(), s=sc.data_ptr(), numel=1, rot=256, d=descs, nl=1, o=out.data_ptr(),
                                  os=out_s.data_ptr(), n=n, k=k, ws=ws.data_ptr(), wsb=ws.numel()), **kw)
    call = lambda a: L.h3q_lora_merge_i8(a["w"], a["s"], a["numel"], a["rot"], a["d"], a["nl"], a["o"], a["os"],
                                         a["n"], a["k"], a["ws"], a["wsb"], st)
    assert call(args(rot=128)) == h3q.ERR_UNSUPPORTED
    assert call(args(k=k - 64)) == h3q.ERR_ARG                      # ConvRot group does not divide k
    assert call(args(os=sc.data_ptr())) == h3q.ERR_ARG              # per-row scales over a scalar input scale
    assert call(args(numel=7)) == h3q.ERR_ARG
    assert call(args(nl=17)) == h3q.ERR_UNSUPPORTED
    assert call(args(ws=ws.data_ptr() + 16)) == h3q.ERR_ARG         # unaligned workspace
    bad = (h3q.LoraDesc * 1)()
    bad[0] = h3q.LoraDesc(descs[0].a, descs[0].b, 4, 9, 1.0)
    assert call(args(d=bad)) == h3q.ERR_ARG                          # factor dtype
    out.fill_(5)
    assert call(args(nl=0)) == h3q.OK                                # nothing to merge: nothing written
    torch.cuda.synchronize()
    assert bool((out == 5).all())
    assert call(args()) == h3q.OK
    torch.cuda.synchronize()
    qo, so = O.lora_merge_i8(q, s, _np_loras(dl), 256)
    assert np.array_equal(out.cpu().numpy(), qo) and np.array_equal(out_s.cpu().numpy(), so)
    del keep


def test_merged_layer_from_files_runs_the_int8_gemm(cuda, tmp_path):
    """A checkpoint layer and a LoRA file, merged through apply_lora (dit.rs:654-690, :599-611), then run: the
    output equals the same GEMM over the oracle's merged codes and scales, bit for bit."""
    pytest.importorskip("safetensors")
    from h3q import checkpoint as C
    from tests.test_checkpoint import PFX, make_checkpoint
    from tests.test_oracle_lora import write_lora
    ck = tmp_path / "model.safetensors"
    tensors = make_checkpoint(ck, seed=4)
    lp = tmp_path / "lora.safetensors"
    write_lora(lp, 512, 256, 8, seed=5, module="blocks.0.attn.qkv", alpha=4.0)
    with C.SafeFile(ck) as f:
        layer = C.load_qlinear(f, "blocks.0.attn.qkv", cuda)
    with C.LoraFile(str(lp)) as lf:
        d = lf.delta("blocks.0.attn.qkv", cuda)
        merged, skipped = C.apply_lora({"blocks.0.attn.qkv": layer}, lf, 0.8, cuda)
    assert merged == ["blocks.0.attn.qkv"] and skipped == []
    q = tensors[PFX + "blocks.0.attn.qkv.weight"].numpy()
    s = tensors[PFX + "blocks.0.attn.qkv.weight_scale"].numpy()
    qo, so = O.lora_merge_i8(q, s, [(d.a.float().cpu().numpy(), d.b.float().cpu().numpy(), d.scale * 0.8)], 256)
    assert np.array_equal(layer.weight.cpu().numpy(), qo)
    assert np.array_equal(layer.scale.cpu().numpy(), so)
    x = (torch.randn((200, 256), device=cuda) * 2).to(torch.bfloat16)
    b = tensors[PFX + "blocks.0.attn.qkv.bias"].to(cuda)
    direct = h3q.QLinear(torch.from_numpy(qo).to(cuda), torch.from_numpy(so).to(cuda), b, convrot=256)
    assert torch.equal(layer.forward(x).view(torch.int16), direct.forward(x).view(torch.int16))
    assert h3q.device_status() == 0
