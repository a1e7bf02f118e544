"""CPU tests of the C ABI: the library loads, exports every function include/h3q.h declares, and its host-side
argument checks (the reference's `bail!`s) answer before any device work.  No GPU calls."""
import ctypes
import os
import re

import pytest

import h3q

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "h3q.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(h3q_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_op_api():
    names = declared_functions()
    for expected in ("h3q_gemm_s8", "h3q_int8_linear_ex", "h3q_quant_rows_i8", "h3q_dequant_i8",
                     "h3q_dequant_nvfp4", "h3q_gate_add", "h3q_available_arch", "h3q_can_fuse_rotation"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(h3q.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) <= set(h3q.SIGNATURES), "python binding misses a declared symbol"


def test_can_fuse_rotation_mirrors_reference_gate():
    assert h3q.can_fuse_rotation(5120, 256)
    assert h3q.can_fuse_rotation(16384, 256)
    assert not h3q.can_fuse_rotation(16640, 256)
    assert not h3q.can_fuse_rotation(5000, 256)
    assert not h3q.can_fuse_rotation(5120, 64)


def test_workspace_size():
    assert h3q.lib().h3q_gemm_s8_workspace_size(3, 1024) == 3072 + 12
    assert h3q.lib().h3q_gemm_s8_workspace_size(3, 1000) == 3072 + 12
    assert h3q.lib().h3q_gemm_s8_workspace_size(32760, 5120) >= 32760 * 5120 + 4 * 32760


def test_gemm_s8_rejects_k_not_multiple_of_64():
    """attn8.rs:571-573: "gemm_s8: bf16 input with K % 64 == 0 required"."""
    L = h3q.lib()
    st = L.h3q_gemm_s8(None, None, None, 1, None, None, 4, 128, 100, 0, 0, None, 0, None)
    assert st == h3q.ERR_ARG
    assert "K % 64 == 0" in h3q.last_error()


def test_gemm_s8_rejects_odd_swiglu_and_short_workspace():
    L = h3q.lib()
    assert L.h3q_gemm_s8(None, None, None, 1, None, None, 4, 127, 128, 1, 0, None, 0, None) == h3q.ERR_ARG
    assert L.h3q_gemm_s8(None, None, None, 1, None, None, 4, 128, 128, 0, 0, None, 10, None) == h3q.ERR_WORKSPACE


def test_int8_linear_ex_shape_checks():
    """kernels.rs:977 "bad shapes" (k % 4) and kernels.rs:1062 (output width % 4)."""
    L = h3q.lib()
    assert L.h3q_int8_linear_ex(None, 2, None, None, 1, None, None, 2, 4, 128, 130, 0, 0, None, 0, None) == h3q.ERR_ARG
    assert "bad shapes" in h3q.last_error()
    assert L.h3q_int8_linear_ex(None, 2, None, None, 1, None, None, 2, 4, 6, 128, 0, 0, None, 0, None) == h3q.ERR_ARG
    assert "multiple of 4" in h3q.last_error()
    assert L.h3q_int8_linear_ex(None, 5, None, None, 1, None, None, 2, 4, 8, 128, 0, 0, None, 0, None) == h3q.ERR_ARG


def test_quant_rows_rotation_checks():
    L = h3q.lib()
    assert L.h3q_quant_rows_i8(None, 2, None, None, 4, 300, 1, None) == h3q.ERR_ARG
    assert "does not divide" in h3q.last_error()
    assert L.h3q_quant_rows_i8(None, 2, None, None, 4, 256 * 65, 1, None) == h3q.ERR_UNSUPPORTED


def test_empty_shapes_are_no_ops():
    L = h3q.lib()
    assert L.h3q_gemm_s8(None, None, None, 1, None, None, 0, 128, 128, 0, 0, None, 0, None) == h3q.OK
    assert L.h3q_quant_rows_i8(None, 2, None, None, 0, 256, 1, None) == h3q.OK
    assert L.h3q_dequant_i8(None, None, 1, None, 2, 0, 16, None) == h3q.OK


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(h3q, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(h3q, "_LIB", None)
    with pytest.raises(RuntimeError, match="not built"):
        h3q.lib()


def test_init_rejects_a_missing_or_unsupported_device():
    """h3q_init on a device index that is no sm_100 GPU (every index on a CPU-only host) fails cleanly."""
    import h3q
    assert h3q.lib().h3q_init(4096) == h3q.ERR_UNSUPPORTED
    assert "not an sm_100 GPU" in h3q.last_error()


def test_host_pipeline_slot_counts_are_checked():
    """h3q_host_pipeline_create_ex rejects fewer than two buffers per direction before touching the device."""
    L = h3q.lib()
    h = ctypes.c_void_p()
    for ins, outs in ((1, 2), (2, 1), (2, 5000)):
        assert L.h3q_host_pipeline_create_ex(256, 1024, 1024, ins, outs, ctypes.byref(h)) == h3q.ERR_ARG
        assert not h.value


def test_host_pipeline_run_argument_checks():
    """h3q_host_pipeline_run rejects a null pipeline before touching the device, and its item layout matches
    include/h3q.h (eleven fields, 8-byte aligned, two trailing ints)."""
    L = h3q.lib()
    item = h3q.HostLinear()
    assert L.h3q_host_pipeline_run(None, ctypes.byref(item), 1, None) == h3q.ERR_ARG
    assert ctypes.sizeof(h3q.HostLinear) == 9 * 8 + 2 * 4
    assert h3q.HostLinear.rotate.offset == 9 * 8 + 4


def test_nsplit_range_matches_python_split():
    from h3q import parallel as P
    L = h3q.lib()
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    for n, g in ((15360, 8), (5120, 3), (600, 2), (100, 4), (13824, 8), (5120, 8)):
        for r in range(g):
            L.h3q_nsplit_range(n, g, r, ctypes.byref(lo), ctypes.byref(hi))
            assert (lo.value, hi.value) == P.nsplit_range(n, g, r)
    L.h3q_nsplit_range(100, 4, 7, ctypes.byref(lo), ctypes.byref(hi))
    assert (lo.value, hi.value) == (0, 0)


def test_nsplit_workspace_and_comm_argument_checks():
    L = h3q.lib()
    # the NCCL form gathers [g][m][widest block] next to its own packed block; the other forms need none
    assert L.h3q_gemm_s8_nsplit_workspace_size(1000, 15360, 8, 2) == 1000 * 2048 * 2 * 9
    assert L.h3q_gemm_s8_nsplit_workspace_size(1000, 15360, 8, 0) == 0
    assert L.h3q_gemm_s8_nsplit_workspace_size(1000, 15360, 8, 1) == 0
    comm = ctypes.c_void_p()
    idb = (ctypes.c_uint8 * 128)()
    assert L.h3q_comm_init(0, 0, idb, ctypes.byref(comm)) == h3q.ERR_ARG and not comm.value
    assert L.h3q_comm_init(2, 2, idb, ctypes.byref(comm)) == h3q.ERR_ARG
    assert L.h3q_gemm_s8_nsplit(None, 0, None, None, None, None, 1, None, None, 1, 8, 16, None, 0, None) == h3q.ERR_ARG
    assert L.h3q_comm_rank(None) == -1 and L.h3q_comm_size(None) == 0
    assert L.h3q_comm_destroy(None) == h3q.OK
