"""h3q.checkpoint -- ComfyUI safetensors checkpoints through the library's native reader (h3q_checkpoint_*).

SafeFile mirrors weights.rs's SafeFile (weights.rs:23-139): names without the "model.diffusion_model." prefix,
shapes, dtypes, metadata and the `<prefix>.comfy_quant` record; tensors come back as numpy arrays (read) or as
torch tensors on a device (load, through pinned staging on the current stream).  load_qlinear is QLinear::load
(weights.rs:493-534): it reads the layer's format and returns an int8 layer (h3q.QLinear), an NVFP4 layer or a
dense one, optionally with the SwiGLU (gate, up) row interleave (weights.rs:765-800) applied during the upload.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import FMT_DENSE, FMT_INT8, FMT_NVFP4, H3QError, QLinear, _stream, check, lib
from . import lora_merge_dense as _lora_merge_dense
from . import nvfp4_linear as _nvfp4_linear

DT_F32, DT_F16, DT_BF16, DT_I8, DT_U8, DT_F8_E4M3, DT_BOOL, DT_I32, DT_I64, DT_F64 = range(10)
DTYPE_NAMES = {DT_F32: "F32", DT_F16: "F16", DT_BF16: "BF16", DT_I8: "I8", DT_U8: "U8", DT_F8_E4M3: "F8_E4M3",
               DT_BOOL: "BOOL", DT_I32: "I32", DT_I64: "I64", DT_F64: "F64"}
# numpy storage of each dtype: bf16 as its uint16 bit patterns, fp8 / bool as bytes (the reference keeps int8 and
# fp8 as raw bytes too, weights.rs:99-112)
_NP = {DT_F32: np.float32, DT_F16: np.float16, DT_BF16: np.uint16, DT_I8: np.int8, DT_U8: np.uint8,
       DT_F8_E4M3: np.uint8, DT_BOOL: np.uint8, DT_I32: np.int32, DT_I64: np.int64, DT_F64: np.float64}


class QLinearSpec(ctypes.Structure):
    """h3q_qlinear_spec."""
    _fields_ = [("format", ctypes.c_int), ("convrot", ctypes.c_int), ("out_features", ctypes.c_int64),
                ("in_features", ctypes.c_int64), ("weight_dtype", ctypes.c_int), ("scale_dtype", ctypes.c_int),
                ("scale_numel", ctypes.c_int64), ("has_bias", ctypes.c_int), ("has_pre_quant_scale", ctypes.c_int)]


def _torch_dtype(dt: int):
    import torch
    return {DT_F32: torch.float32, DT_F16: torch.float16, DT_BF16: torch.bfloat16, DT_I8: torch.int8,
            DT_U8: torch.uint8, DT_F8_E4M3: torch.uint8, DT_BOOL: torch.uint8, DT_I32: torch.int32,
            DT_I64: torch.int64, DT_F64: torch.float64}[dt]


def interleave_rows(a):
    """interleave_rows (weights.rs:679-687): rows [g_0 .. g_{n/2-1}, u_0 .. u_{n/2-1}] -> [g_0, u_0, g_1, u_1, ...]
    (numpy or torch, first dimension even)."""
    n = a.shape[0]
    if n % 2:
        raise ValueError("interleave_rows: the first dimension must be even")
    return a.reshape((2, n // 2) + tuple(a.shape[1:])).swapaxes(0, 1).reshape(a.shape)


class SafeFile:
    """A safetensors checkpoint opened by the native reader."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        check(lib().h3q_checkpoint_open(str(path).encode(), ctypes.byref(h)))
        self._h = h
        self.path = str(path)

    def close(self) -> None:
        if self._h:
            lib().h3q_checkpoint_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list[str]:
        return [lib().h3q_checkpoint_name(self._h, i).decode() for i in range(lib().h3q_checkpoint_count(self._h))]

    def names_with_prefix(self, prefix: str) -> list[str]:
        return [n for n in self.names() if n.startswith(prefix)]

    def has(self, name: str) -> bool:
        return bool(lib().h3q_checkpoint_has(self._h, name.encode()))

    def metadata(self, key: str) -> str | None:
        v = lib().h3q_checkpoint_metadata(self._h, key.encode())
        return None if v is None else v.decode()

    def info(self, name: str):
        """(dtype name, shape tuple, bytes)."""
        dt, nd, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        shape = (ctypes.c_int64 * 8)()
        check(lib().h3q_checkpoint_info(self._h, name.encode(), ctypes.byref(dt), ctypes.byref(nd), shape,
                                        ctypes.byref(nb)))
        return DTYPE_NAMES[dt.value], tuple(shape[i] for i in range(nd.value)), nb.value

    def _dt(self, name: str) -> int:
        d = {v: k for k, v in DTYPE_NAMES.items()}
        return d[self.info(name)[0]]

    def read(self, name: str) -> np.ndarray:
        """The tensor in its storage dtype, on the host."""
        _, shape, nbytes = self.info(name)
        out = np.empty(nbytes, dtype=np.uint8)
        check(lib().h3q_checkpoint_read(self._h, name.encode(), out.ctypes.data_as(ctypes.c_void_p), nbytes))
        return out.view(_NP[self._dt(name)]).reshape(shape if shape else (1,))

    def load(self, name: str, device, interleave: bool = False):
        """SafeFile::load (weights.rs:114-119): the tensor in its storage dtype on `device` (scalars as [1]);
        interleave=True lands the two halves of the first dimension as (gate, up) row pairs."""
        import torch
        _, shape, nbytes = self.info(name)
        if torch.device(device).type != "cuda":  # host tensors: pread, no copy engine
            a = self.read(name)
            if interleave:
                a = interleave_rows(a)
            return torch.from_numpy(np.ascontiguousarray(a)).view(_torch_dtype(self._dt(name)))
        t = torch.empty(shape if shape else (1,), dtype=_torch_dtype(self._dt(name)), device=device)
        check(lib().h3q_checkpoint_upload(self._h, name.encode(), ctypes.c_void_p(t.data_ptr()), nbytes,
                                          int(interleave), _stream(t.device)))
        return t

    def load_as(self, name: str, device, dtype):
        return self.load(name, device).to(dtype)

    def comfy_quant(self, prefix: str):
        """The parsed `<prefix>.comfy_quant` record, or None (SafeFile::comfy_quant, weights.rs:130-137)."""
        key = f"{prefix}.comfy_quant"
        if not self.has(key):
            return None
        return json.loads(self.read(key).tobytes())

    def qlinear_spec(self, prefix: str) -> QLinearSpec:
        spec = QLinearSpec()
        check(lib().h3q_checkpoint_qlinear(self._h, prefix.encode(), ctypes.byref(spec)))
        return spec


class Nvfp4Linear:
    """QFormat::Nvfp4 layer: packed e2m1 weight, e4m3 block scales, f32 global scale, optional AWQ scale and bias;
    forward is QLinear::apply's NVFP4 branch (h3q_nvfp4_linear)."""

    def __init__(self, q, block_scale, global_scale, pre_quant_scale=None, bias=None):
        self.q, self.block_scale, self.global_scale = q, block_scale, global_scale
        self.pre_quant_scale, self.bias = pre_quant_scale, bias
        self.out_features, self.in_features = q.shape[0], q.shape[1] * 2

    def forward(self, x):
        return _nvfp4_linear(x, self.q, self.block_scale, self.global_scale, self.pre_quant_scale, self.bias)


class DenseLinear:
    """QFormat::Dense layer (outside the int8 hot path): forward is a plain library matmul, as the reference's
    candle matmul."""

    def __init__(self, weight, bias=None):
        self.weight, self.bias = weight, bias
        self.out_features, self.in_features = weight.shape

    def forward(self, x):
        y = x @ self.weight.to(x.dtype).t()
        return y if self.bias is None else y + self.bias.to(x.dtype)

    def merge_loras(self, loras) -> None:
        """QLinear::merge_loras for a dense layer (weights.rs:710-715), through h3q_lora_merge_dense."""
        if loras:
            self.weight = _lora_merge_dense(self.weight.contiguous(), loras)


def load_qlinear(f: SafeFile, prefix: str, device, compute_dtype=None, interleave_swiglu: bool = False):
    """QLinear::load (weights.rs:493-534) for the layer at `prefix`.  interleave_swiglu applies
    QLinear::interleave_swiglu (weights.rs:765-800) to an int8 layer's weight rows, per-row scales and bias while
    they are uploaded (other formats are returned unchanged, as in the reference)."""
    import torch
    compute_dtype = compute_dtype or torch.bfloat16
    spec = f.qlinear_spec(prefix)
    bias = f.load(f"{prefix}.bias", device).to(torch.float32) if spec.has_bias else None
    if spec.format == FMT_INT8:
        il = bool(interleave_swiglu)
        w = f.load(f"{prefix}.weight", device, interleave=il)
        scale = f.load(f"{prefix}.weight_scale", device).to(torch.float32)
        if il and scale.numel() == spec.out_features:
            scale = f.load(f"{prefix}.weight_scale", device, interleave=True).to(torch.float32)
        if il and bias is not None:
            bias = interleave_rows(bias).contiguous()
        layer = QLinear(w, scale, bias, convrot=spec.convrot, interleaved=il)
        layer.spec = spec
        return layer
    if spec.format == FMT_NVFP4:
        q = f.load(f"{prefix}.weight", device)
        bs = f.load(f"{prefix}.weight_scale", device)
        g = f.load(f"{prefix}.weight_scale_2", device).to(torch.float32).reshape(1)
        pq = f.load(f"{prefix}.pre_quant_scale", device).to(compute_dtype) if spec.has_pre_quant_scale else None
        layer = Nvfp4Linear(q, bs, g, pq, bias)
        layer.spec = spec
        return layer
    if spec.format == FMT_DENSE:
        layer = DenseLinear(f.load(f"{prefix}.weight", device), bias)
        layer.spec = spec
        return layer
    raise H3QError(1, f"{prefix}: unknown format {spec.format}")


class LoraDelta:
    """One layer's low-rank pair (lora.rs:15-23): a [r, in] and b [out, r] as bf16 on the device, scale =
    alpha / rank (1 without an alpha), and the optional `reshape_weight` target shape."""

    def __init__(self, a, b, scale: float, reshape=None):
        self.a, self.b, self.scale, self.reshape = a, b, scale, reshape


class LoraFile:
    """A ComfyUI-style LoRA file for the DiT (lora.rs:11-72): `<module>.lora_B/lora_A.weight` or
    `<module>.lora_up/lora_down.weight`, optional `<module>.alpha` and `<module>.reshape_weight`, all under a
    "diffusion_model." prefix when any name carries it."""

    def __init__(self, path: str):
        self.file = SafeFile(path)
        self.prefix = "diffusion_model." if any(k.startswith("diffusion_model.") for k in self.file.names()) else ""

    def close(self) -> None:
        self.file.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def metadata(self, key: str) -> str | None:
        return self.file.metadata(key)

    def delta(self, module: str, device) -> LoraDelta | None:
        """Lora::delta (lora.rs:42-71): the pair for `module` (a layer name without ".weight"), or None.  The
        factors are loaded as bf16 (lora.rs:51-53) and flattened from dimension 1."""
        import torch
        p = self.prefix + module
        if self.file.has(f"{p}.lora_B.weight"):
            up, down = f"{p}.lora_B.weight", f"{p}.lora_A.weight"
        elif self.file.has(f"{p}.lora_up.weight"):
            up, down = f"{p}.lora_up.weight", f"{p}.lora_down.weight"
        else:
            return None
        b = self.file.load(up, device).to(torch.bfloat16)
        a = self.file.load(down, device).to(torch.bfloat16)
        a = a.reshape(a.shape[0], -1)
        b = b.reshape(b.shape[0], -1)
        rank = float(a.shape[0])
        scale = 1.0
        if self.file.has(f"{p}.alpha"):
            alpha = self.file.load(f"{p}.alpha", "cpu").to(torch.float32).reshape(-1)[0]
            scale = float(alpha) / rank
        reshape = None
        if self.file.has(f"{p}.reshape_weight"):
            reshape = [int(v) for v in self.file.read(f"{p}.reshape_weight").astype(np.int64).reshape(-1)]
        return LoraDelta(a, b, scale, reshape)


def apply_lora(layers: dict, lora: LoraFile, strength: float, device):
    """The DiT's apply_lora + merge (dit.rs:654-690, :599-611) over `layers` (module name -> layer): each layer
    with a matching pair of the right shape gets scale * strength * (b @ a) folded into its weight.  Returns
    (merged, skipped) module names: a pair whose shapes do not match the layer or that carries reshape_weight is
    skipped, as the reference does; NVFP4 layers are skipped too (the reference keeps its LoRAs on a runtime path,
    weights.rs:708, that this library does not serve)."""
    merged, skipped = [], []
    for name, layer in layers.items():
        d = lora.delta(name, device)
        if d is None:
            continue
        out_f = layer.desc.out_features if isinstance(layer, QLinear) else layer.out_features
        in_f = layer.desc.in_features if isinstance(layer, QLinear) else layer.in_features
        if (d.a.shape[1] != in_f or d.b.shape[0] != out_f or d.reshape is not None
                or isinstance(layer, Nvfp4Linear)):
            skipped.append(name)
            continue
        layer.merge_loras([(d.a, d.b, d.scale * strength)])
        merged.append(name)
    return merged, skipped


__all__ = ["SafeFile", "QLinearSpec", "Nvfp4Linear", "DenseLinear", "load_qlinear", "interleave_rows", "DTYPE_NAMES",
           "LoraDelta", "LoraFile", "apply_lora"]
