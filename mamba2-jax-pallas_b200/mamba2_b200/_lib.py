"""ctypes binding of libssd_b200.so (the C ABI in include/ssd_b200.h).

Torch is used only for device memory and the current CUDA stream: tensors are passed
to the library as raw device pointers.  There is no fallback: if the library cannot
be loaded, or a tensor is not on a CUDA device, the call raises.
"""

from __future__ import annotations

import ctypes
import math
import os
import pathlib

import torch

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = pathlib.Path(os.environ.get("SSD_B200_LIB", _HERE / "libssd_b200.so"))

SSD_DTYPE_F32 = 0
SSD_DTYPE_BF16 = 1
SSD_FLAG_FORCE_SIMT = 1
SSD_FLAG_ROUND_STATES = 2
SSD_FLAG_BF16_MMA = 4
SSD_FLAG_TEST_WAIT_TIMEOUT = 8
# the ssd_b200.h these ctypes structures describe
ABI_VERSION = 2
SSD_NOALLOC_SCRATCH_BYTES = 16 << 20

STATUS_NAMES = {0: "SSD_OK", 1: "SSD_ERR_INVALID_ARG", 2: "SSD_ERR_UNSUPPORTED",
                3: "SSD_ERR_ALIGNMENT", 4: "SSD_ERR_WORKSPACE", 5: "SSD_ERR_CUDA",
                6: "SSD_ERR_TIMEOUT"}

# Every symbol include/ssd_b200.h declares (checked by the CPU test suite).
EXPORTED = ["ssd_combined_workspace_bytes", "ssd_combined_uses_tensor_cores",
            "ssd_combined_num_launches", "ssd_combined_fwd", "ssd_combined_fwd_noalloc", "ssd_chunk_cumsum_fwd",
            "ssd_chunk_state_fwd", "ssd_state_passing_fwd", "ssd_bmm_chunk_fwd",
            "ssd_chunk_scan_fwd", "ssd_chunk_state_varlen_fwd", "ssd_selective_state_update",
            "ssd_causal_conv1d_fwd", "ssd_causal_conv1d_update", "ssd_rms_norm_gated", "ssd_sp_state_fixup", "ssd_status_copy_async", "ssd_status_decode",
            "ssd_last_error", "ssd_abi_version", "ssd_set_fp32_stage_path"]

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float


class SsdFwdParams(ctypes.Structure):
    _fields_ = [("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64),
                ("ngroups", _i64), ("dstate", _i64), ("chunk_size", _i64),
                ("dtype", _i32), ("dt_dtype", _i32), ("dt_softplus", _i32), ("D_ndim", _i32),
                ("dt_min", _f32), ("dt_max", _f32), ("num_seqs", _i32), ("flags", _i32),
                ("x", _vp), ("dt", _vp), ("A", _vp), ("B", _vp), ("C", _vp), ("D", _vp),
                ("z", _vp), ("dt_bias", _vp), ("initial_states", _vp), ("seq_idx", _vp),
                ("cu_seqlens", _vp),
                ("out", _vp), ("out_x", _vp), ("final_states", _vp), ("varlen_states", _vp),
                ("dA_cumsum", _vp), ("dt_out", _vp)]


class SsuParams(ctypes.Structure):
    _fields_ = [("batch", _i64), ("nheads", _i64), ("headdim", _i64), ("ngroups", _i64),
                ("dstate", _i64), ("dtype", _i32), ("dt_dtype", _i32), ("dt_ndim", _i32),
                ("A_ndim", _i32), ("D_ndim", _i32), ("dt_bias_ndim", _i32),
                ("dt_softplus", _i32), ("reserved", _i32),
                ("state", _vp), ("x", _vp), ("dt", _vp), ("A", _vp), ("B", _vp), ("C", _vp),
                ("D", _vp), ("z", _vp), ("dt_bias", _vp), ("out", _vp)]


class Conv1dParams(ctypes.Structure):
    _fields_ = [("batch", _i64), ("dim", _i64), ("seqlen", _i64),
                ("x_stride_b", _i64), ("x_stride_d", _i64), ("x_stride_t", _i64),
                ("out_stride_b", _i64), ("out_stride_d", _i64), ("out_stride_t", _i64),
                ("width", _i32), ("dtype", _i32), ("out_dtype", _i32), ("silu", _i32),
                ("x", _vp), ("weight", _vp), ("bias", _vp), ("seq_idx", _vp), ("out", _vp),
                ("weight_dtype", _i32), ("bias_dtype", _i32)]


class Conv1dUpdateParams(ctypes.Structure):
    _fields_ = [("batch", _i64), ("dim", _i64), ("state_stride_b", _i64), ("state_stride_d", _i64),
                ("width", _i32), ("x_dtype", _i32), ("state_dtype", _i32), ("out_dtype", _i32),
                ("silu", _i32), ("reserved", _i32),
                ("x_new", _vp), ("conv_state", _vp), ("weight", _vp), ("bias", _vp), ("out", _vp),
                ("weight_dtype", _i32), ("bias_dtype", _i32)]


class RmsNormParams(ctypes.Structure):
    _fields_ = [("rows", _i64), ("hidden", _i64), ("group_size", _i64),
                ("x_stride_row", _i64), ("z_stride_row", _i64), ("out_stride_row", _i64),
                ("x_dtype", _i32), ("z_dtype", _i32), ("weight_dtype", _i32), ("out_dtype", _i32),
                ("norm_before_gate", _i32), ("eps", _f32),
                ("x", _vp), ("z", _vp), ("weight", _vp), ("out", _vp)]


class SpFixupParams(ctypes.Structure):
    _fields_ = [("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64),
                ("ngroups", _i64), ("dstate", _i64), ("chunk_size", _i64),
                ("dtype", _i32), ("reserved", _i32),
                ("C", _vp), ("z", _vp), ("dA_cumsum", _vp), ("state_in", _vp), ("carried_len", _vp),
                ("out", _vp), ("final_states", _vp)]


class SsdError(RuntimeError):
    """A non-zero ssd_status_t from the library."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and type the shared library.  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} not found: build it with "
                           f"`python mamba2-jax-pallas_b200/build.py` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.POINTER
    lib.ssd_last_error.restype = ctypes.c_char_p
    lib.ssd_abi_version.restype = ctypes.c_int
    lib.ssd_combined_workspace_bytes.argtypes = [P(SsdFwdParams)]
    lib.ssd_combined_workspace_bytes.restype = ctypes.c_size_t
    lib.ssd_combined_uses_tensor_cores.argtypes = [P(SsdFwdParams)]
    lib.ssd_combined_num_launches.argtypes = [P(SsdFwdParams)]
    lib.ssd_combined_fwd.argtypes = [P(SsdFwdParams), _vp, ctypes.c_size_t, _vp]
    lib.ssd_combined_fwd_noalloc.argtypes = [P(SsdFwdParams), _vp]
    lib.ssd_chunk_cumsum_fwd.argtypes = [_vp, _i32, _vp, _vp, _i32, _f32, _f32, _i64, _i64, _i64,
                                         _i64, _vp, _vp, _vp]
    lib.ssd_chunk_state_fwd.argtypes = [_vp, _vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                        _i64, _i64, _i64, _vp, _vp]
    lib.ssd_state_passing_fwd.argtypes = [_vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64,
                                          _i64, _i64, _vp, _i32, _vp, _vp]
    lib.ssd_bmm_chunk_fwd.argtypes = [_vp, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64,
                                      _vp, _vp]
    lib.ssd_chunk_scan_fwd.argtypes = [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp,
                                       _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp,
                                       _vp]
    lib.ssd_causal_conv1d_fwd.argtypes = [P(Conv1dParams), _vp]
    lib.ssd_causal_conv1d_update.argtypes = [P(Conv1dUpdateParams), _vp]
    lib.ssd_rms_norm_gated.argtypes = [P(RmsNormParams), _vp]
    lib.ssd_sp_state_fixup.argtypes = [P(SpFixupParams), _vp]
    lib.ssd_chunk_state_varlen_fwd.argtypes = [_vp, _vp, _i32, _vp, _vp, _vp, _i32, _vp, _i32,
                                               _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp]
    lib.ssd_selective_state_update.argtypes = [P(SsuParams), _vp]
    lib.ssd_status_copy_async.argtypes = [_vp, _vp, _vp]
    lib.ssd_status_decode.argtypes = [ctypes.c_uint32]
    lib.ssd_set_fp32_stage_path.argtypes = [_i32]
    for name in EXPORTED:
        if name not in ("ssd_last_error", "ssd_abi_version", "ssd_combined_workspace_bytes"):
            getattr(lib, name).restype = ctypes.c_int
    if lib.ssd_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libssd_b200.so has ABI version {lib.ssd_abi_version()}, these bindings "
                           f"describe version {ABI_VERSION}: rebuild the library")
    _lib = lib
    return lib


def check(code: int) -> None:
    if code != 0:
        msg = load().ssd_last_error().decode(errors="replace")
        raise SsdError(code, msg)


FP32_STAGES_TENSOR_CORES = 0
FP32_STAGES_CUDA_CORES = 1


class fp32_stage_path:
    """Choose the kernels behind chunk_state, bmm_chunk and chunk_scan for fp32 inputs
    (process-wide, ssd_set_fp32_stage_path): FP32_STAGES_TENSOR_CORES (default; split-bf16
    tcgen05 MMAs) or FP32_STAGES_CUDA_CORES (fp32 FFMA).  A context manager that puts the
    previous choice back on exit."""

    def __init__(self, path: int):
        self.path = path
        self.prev = None

    def __enter__(self):
        r = load().ssd_set_fp32_stage_path(self.path)
        if r < 0:
            raise SsdError(1, load().ssd_last_error().decode(errors="replace"))
        self.prev = r
        return self

    def __exit__(self, *exc):
        load().ssd_set_fp32_stage_path(self.prev)
        return False


def check_device_status(workspace: torch.Tensor, stream=None) -> None:
    """Read the device status word of the last ssd_combined_fwd call that used ``workspace``
    (waits for that stream) and raise SsdError if a bounded wait inside the kernel gave up."""
    lib = load()
    s = torch.cuda.current_stream(workspace.device) if stream is None else stream
    word = torch.empty(1, dtype=torch.int32, device=workspace.device)
    check(lib.ssd_status_copy_async(workspace.data_ptr(), word.data_ptr(), s.cuda_stream))
    s.synchronize()
    check(lib.ssd_status_decode(int(word.item()) & 0xFFFFFFFF))


# ---------------------------------------------------------------------------
# tensor helpers
# ---------------------------------------------------------------------------

def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return SSD_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return SSD_DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype} (float32 or bfloat16)")


def torch_dtype(code: int):
    return torch.bfloat16 if code == SSD_DTYPE_BF16 else torch.float32


def dev(t, name: str, dtype=None):
    """Contiguous CUDA tensor (optionally cast), or None."""
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the SSD kernels have no CPU path)")
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def limits(dt_limit):
    lo, hi = float(dt_limit[0]), float(dt_limit[1])
    return lo, (hi if math.isfinite(hi) else float("inf"))
