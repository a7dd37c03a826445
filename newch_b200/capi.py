"""ctypes description of the nc.h C ABI (include/nc.h) and of the side API (include/nc_ext.h).

The same table binds the B200 library (newch_b200/libnc.so) and any other library that exports the
newch engine ABI, so one driver can run a workload on either. Struct layouts and argument types
follow the newch engine header (engine/include/nc.h:78-83, :109-114, :123-133, :370-375) and the
newch ctypes surface (newch/_lib.py:19-47, :78-172).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

F32, I32, F16, I8, U8 = 0, 1, 2, 3, 4
DTYPE_SIZE = {F32: 4, I32: 4, F16: 2, I8: 1, U8: 1}
ALL_AXES = -128


class Config(Structure):
    _fields_ = [("arena_chunk_bytes", c_size_t), ("seed", c_uint64), ("force_reference", c_int), ("threads", c_int)]


class CpuInfo(Structure):
    _fields_ = [("arch", c_char_p), ("has_neon", c_int), ("has_dotprod", c_int), ("has_fp16", c_int),
                ("has_avx2", c_int), ("has_fma", c_int), ("has_rvv", c_int), ("n_cores", c_int),
                ("n_big_cores", c_int)]


class MemStats(Structure):
    _fields_ = [("persistent_bytes", c_size_t), ("arena_bytes_in_use", c_size_t),
                ("arena_bytes_reserved", c_size_t), ("arena_peak_bytes", c_size_t)]


class OptimOpts(Structure):
    _fields_ = [(n, c_float) for n in ("lr", "momentum", "weight_decay", "beta1", "beta2", "eps")]


P = c_void_p
I64P = POINTER(c_int64)
PP = POINTER(c_void_p)
SCALAR_FN = ctypes.CFUNCTYPE(c_void_p, c_void_p, PP, c_void_p)

# name -> (restype, argtypes).  Every NC_API function of include/nc.h.
SIGNATURES: dict = {
    # context
    "nc_init": (P, [POINTER(Config)]),
    "nc_free_ctx": (None, [P]),
    "nc_manual_seed": (None, [P, c_uint64]),
    "nc_step_end": (None, [P]),
    "nc_arena_trim": (None, [P]),
    "nc_num_threads": (c_int, [P]),
    "nc_persistent_begin": (None, [P]),
    "nc_persistent_end": (None, [P]),
    "nc_set_grad_enabled": (c_int, [P, c_int]),
    "nc_ok": (c_int, [P]),
    "nc_status_code": (c_int, [P]),
    "nc_error": (c_char_p, [P]),
    "nc_clear_error": (None, [P]),
    "nc_get_mem_stats": (MemStats, [P]),
    "nc_reset_peak": (None, [P]),
    "nc_cpu": (POINTER(CpuInfo), [P]),
    "nc_kernel_backend": (c_char_p, [P]),
    # tensors
    "nc_empty": (P, [P, c_int, c_int, I64P]),
    "nc_zeros": (P, [P, c_int, c_int, I64P]),
    "nc_full": (P, [P, c_float, c_int, I64P]),
    "nc_randn": (P, [P, c_float, c_int, I64P]),
    "nc_rand_uniform": (P, [P, c_float, c_float, c_int, I64P]),
    "nc_from_data": (P, [P, c_int, c_void_p, c_int, I64P]),
    "nc_scalar": (P, [P, c_float]),
    "nc_parameter": (P, [P, P, c_int, I64P]),
    "nc_ndim": (c_int, [P]),
    "nc_dim": (c_int64, [P, c_int]),
    "nc_shape": (I64P, [P]),
    "nc_numel": (c_int64, [P]),
    "nc_get_dtype": (c_int, [P]),
    "nc_is_contiguous": (c_int, [P]),
    "nc_requires_grad": (c_int, [P]),
    "nc_is_persistent": (c_int, [P]),
    "nc_release": (None, [P]),
    "nc_set_requires_grad": (None, [P, c_int]),
    "nc_grad": (P, [P]),
    "nc_set_name": (None, [P, c_char_p]),
    "nc_name": (c_char_p, [P]),
    "nc_data_f32": (c_void_p, [P]),
    "nc_data_i32": (c_void_p, [P]),
    "nc_item": (c_float, [P]),
    "nc_get": (c_float, [P, I64P]),
    "nc_copy_to": (c_int, [P, c_void_p, c_size_t]),
    "nc_copy_from": (c_int, [P, c_void_p, c_size_t]),
    "nc_print": (None, [P]),
    # ops
    **{f"nc_{n}": (P, [P, P]) for n in ("add", "sub", "mul", "div", "matmul", "cross_entropy", "mse_loss",
                                         "index_select")},
    **{f"nc_{n}": (P, [P]) for n in ("neg", "exp", "log", "sqrt", "relu", "sigmoid", "tanh", "contiguous",
                                      "log_softmax", "softmax", "detach", "relu6", "hardsigmoid", "hardswish",
                                      "silu")},
    **{f"nc_{n}": (P, [P, c_float]) for n in ("scale", "add_scalar", "pow_scalar", "leaky_relu", "dropout")},
    **{f"nc_{n}": (P, [P, c_int, c_int]) for n in ("sum", "mean", "max", "transpose")},
    "nc_gelu": (P, [P, c_int]),
    "nc_linear_fn": (P, [P, P, P]),
    "nc_argmax": (P, [P, c_int]),
    "nc_reshape": (P, [P, c_int, I64P]),
    "nc_slice": (P, [P, c_int, c_int64, c_int64, c_int64]),
    "nc_conv2d": (P, [P, P, P, c_int, c_int, c_int, c_int]),
    "nc_conv2d_ex": (P, [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "nc_max_pool2d": (P, [P, c_int, c_int, c_int, c_int, c_int, c_int]),
    "nc_avg_pool2d": (P, [P, c_int, c_int, c_int, c_int, c_int, c_int]),
    "nc_batch_norm": (P, [P, P, P, P, P, c_int, c_float, c_float]),
    "nc_layer_norm": (P, [P, c_int, P, P, c_float]),
    "nc_masked_fill": (P, [P, P, c_float]),
    "nc_nll_loss": (P, [P, P, c_int]),
    "nc_compare": (P, [P, P, c_int]),
    "nc_cat": (P, [c_int, PP, c_int]),
    "nc_to_dtype": (P, [P, c_int]),
    # quantization
    "nc_quantize_rows": (P, [P, PP]),
    "nc_linear_int8": (P, [P, P, P, P]),
    # serialization
    "nc_save": (c_int, [P, c_char_p, c_int, POINTER(c_char_p), PP]),
    "nc_load": (c_int, [P, c_char_p, c_int, POINTER(c_char_p), PP]),
    # autograd
    "nc_backward": (c_int, [P]),
    "nc_backward_ex": (c_int, [P, c_int, PP, c_int]),
    "nc_release_temp": (None, [P]),
    "nc_zero_grad": (None, [P]),
    "nc_clear_grad": (None, [P]),
    "nc_gradcheck": (c_float, [P, SCALAR_FN, PP, c_int, c_void_p, c_float]),
    # C-side modules
    "nc_linear": (P, [P, c_int64, c_int64, c_int]),
    "nc_act": (P, [P, c_int]),
    "nc_sequential": (P, [P, c_int, PP]),
    "nc_forward": (P, [P, P]),
    "nc_parameters": (c_int, [P, PP, c_int]),
    "nc_module_name": (c_char_p, [P]),
    "nc_set_training": (None, [P, c_int]),
    # optimizers
    "nc_sgd": (P, [P, PP, c_int, OptimOpts]),
    "nc_adam": (P, [P, PP, c_int, OptimOpts]),
    "nc_adamw": (P, [P, PP, c_int, OptimOpts]),
    "nc_rmsprop": (P, [P, PP, c_int, OptimOpts, c_int]),
    "nc_optim_zero_grad": (None, [P]),
    "nc_optim_clear_grad": (None, [P]),
    "nc_optim_step": (None, [P]),
    "nc_optim_free": (None, [P]),
    "nc_optim_set_lr": (None, [P, c_float]),
    "nc_optim_state": (c_void_p, [P, c_int, c_int]),
    "nc_optim_get_step": (c_int64, [P]),
    "nc_optim_set_step": (None, [P, c_int64]),
    "nc_optim_set_opts": (None, [P, OptimOpts]),
    "nc_optim_set_accumulation": (None, [P, c_int]),
    "nc_clip_grad_norm": (c_float, [PP, c_int, c_float]),
}

# Side API of the B200 build (include/nc_ext.h): device selection, data-parallel set-up and
# counters. Absent from other engines.
EXT_SIGNATURES: dict = {
    "nc_ext_device_count": (c_int, []),
    "nc_ext_device_name": (c_char_p, [P]),
    "nc_ext_synchronize": (c_int, [P]),
    "nc_ext_pipeline_wait_probe": (c_int, [P]),
    "nc_ext_launch_count": (c_int64, [P]),
    "nc_ext_gemm_mode": (c_char_p, [P]),
    "nc_ext_nccl_unique_id": (c_int, [c_void_p, c_int]),
    "nc_ext_dp_init": (c_int, [P, c_int, c_int, c_void_p, c_int]),
    "nc_ext_dp_world": (c_int, [P]),
    "nc_ext_dp_rng_stride": (c_int, [P, c_int64]),
    "nc_ext_rng_position": (c_int64, [P]),
    "nc_ext_stream": (c_void_p, [P]),
    "nc_ext_timing": (c_int, [P, c_int]),
    "nc_ext_kernel_time": (c_int, [P, c_char_p, POINTER(ctypes.c_double), POINTER(c_int64)]),
    "nc_ext_kernel_entry": (c_int, [P, c_int, POINTER(c_char_p), POINTER(ctypes.c_double), POINTER(c_int64),
                                    POINTER(ctypes.c_double), POINTER(ctypes.c_double)]),
    "nc_ext_timing_reset": (None, [P]),
    "nc_ext_cross_entropy_fwd_noalloc": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                                 c_void_p]),
}


def kernel_table(lib, ctx) -> list:
    """[(name, ms, launches, flops, bytes)] of the timed kernel classes (timing must be on)."""
    out, i = [], 0
    name, ms, cnt = c_char_p(), ctypes.c_double(), c_int64()
    fl, by = ctypes.c_double(), ctypes.c_double()
    while lib.nc_ext_kernel_entry(ctx, i, ctypes.byref(name), ctypes.byref(ms), ctypes.byref(cnt), ctypes.byref(fl),
                                  ctypes.byref(by)):
        out.append((name.value.decode(), ms.value, cnt.value, fl.value, by.value))
        i += 1
    return out

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent


def b200_library_path() -> Path:
    return PKG_DIR / "libnc.so"


def load(path, ext: bool = False) -> ctypes.CDLL:
    """Opens an nc-ABI library and applies the signature table. ``ext`` also binds nc_ext_*."""
    path = Path(path)
    if not path.exists():
        raise OSError(f"nc library not found: {path} (run __graft_entry__.build() or make -C newch_b200/csrc)")
    lib = ctypes.CDLL(str(path), mode=os.RTLD_LOCAL)
    table = dict(SIGNATURES)
    if ext:
        table.update(EXT_SIGNATURES)
    for name, (res, args) in table.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def load_b200() -> ctypes.CDLL:
    """The B200 engine. Raises if it was not built: there is no fallback."""
    return load(b200_library_path(), ext=True)


def shape_arg(shape):
    shape = tuple(int(s) for s in shape)
    return len(shape), (c_int64 * max(len(shape), 1))(*shape)


def ptr_array(ptrs):
    ptrs = list(ptrs)
    return (c_void_p * max(len(ptrs), 1))(*ptrs)
