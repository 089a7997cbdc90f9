"""ctypes bindings of libkmamba_b200.so for the tests and bench.py.

The library is the product: a C host layer over sm_100a kernels exposing
the k-mamba C API (scan.h, scan_nd.h, convnd.h, wavefront_plan.h, ...) and
the batched kmb_* extensions (kmamba_b200.h).  This module only declares
the C structs and prototypes so Python can call them; it computes nothing.

Pointers are passed as integers: ``tensor.data_ptr()`` for torch tensors
(device or host) or ``array.ctypes.data`` for numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkmamba_b200.so")

KMB_OK = 0
KMB_EINVAL = -1
KMB_ECUDA = -2
KMB_ENOMEM = -3
KMB_ETIMEOUT = -4
KMB_EUNSUPPORTED = -5

KMB_SCAN1D_CHUNK = 8

fp = C.c_void_p  # float* / long* passed as raw addresses
lg = C.c_long


class ScanParams(C.Structure):
    _fields_ = [(n, fp) for n in ("x", "A", "B", "C", "delta", "h", "y")] + [
        ("L", lg), ("D", lg), ("M", lg)]


class ScanBackwardParams(C.Structure):
    _fields_ = [(n, fp) for n in ("x", "A", "B", "C", "delta", "h0", "h", "dy", "dx",
                                  "dA", "dB", "dC", "ddelta")] + [
        ("L", lg), ("D", lg), ("M", lg)]


class ScanBackwardSharedParams(C.Structure):
    _fields_ = [(n, fp) for n in ("x", "A", "A_diag", "B", "C", "delta", "h0", "h", "dy",
                                  "dx", "dA", "dB", "dC", "ddelta")] + [
        ("L", lg), ("D", lg)]


class Scan2DParams(C.Structure):
    _fields_ = [(n, fp) for n in ("x", "A1", "A2", "B", "C", "delta1", "delta2", "h", "y")] + [
        ("d1", lg), ("d2", lg), ("D", lg), ("M", lg)]


class ScanNDParams(C.Structure):
    _fields_ = [("dims", fp), ("ndims", lg), ("D", lg), ("M", lg)] + [
        (n, fp) for n in ("x", "A", "B", "C", "delta", "h", "y", "theta", "lambda_")]


class ConvNDParams(C.Structure):
    _fields_ = [(n, fp) for n in ("input", "kernel", "bias", "output", "dy", "dinput",
                                  "dkernel", "dbias", "dims")] + [
        ("ndims", lg), ("D", lg), ("K", lg)]


class KMWavefrontPlan(C.Structure):
    _fields_ = [("dims", C.POINTER(lg)), ("ndims", lg), ("total_points", lg),
                ("max_level", lg), ("max_level_size", lg),
                ("level_starts", C.POINTER(lg)), ("level_offsets", C.POINTER(lg))]


class KmbGemm(C.Structure):
    _fields_ = [(n, fp) for n in ("A", "B", "C", "bias", "residual")] + [
        (n, lg) for n in ("M", "N", "K", "lda", "ldb", "ldc", "ldr")] + [
        (n, C.c_int) for n in ("a_mn_major", "b_mn_major", "c_bf16", "act", "accumulate",
                               "pad_")]


class KMambaDistributedConfig(C.Structure):
    _fields_ = [("world_size", C.c_int), ("rank", C.c_int), ("local_rank", C.c_int),
                ("layer_start", C.c_size_t), ("layer_end", C.c_size_t),
                ("batch_start", C.c_size_t), ("batch_end", C.c_size_t),
                ("use_nccl", C.c_int), ("use_p2p", C.c_int)]


class KMambaDistributedContext(C.Structure):
    _fields_ = [("config", KMambaDistributedConfig), ("nccl_comm", C.c_void_p),
                ("stream", C.c_void_p), ("nccl_scratch", C.c_void_p),
                ("scratch_size", C.c_size_t)]


class KmbNDModelConfig(C.Structure):
    _fields_ = [("dims", lg * 3), ("dim", lg), ("n_layers", lg), ("vocab", lg),
                ("seed", C.c_ulonglong), ("micro_batch", lg)]


class KmbScan1D(C.Structure):
    _fields_ = [(n, fp) for n in ("x", "dt", "A", "B", "C", "h0", "y", "h_last", "h_all",
                                  "ckpt", "dy", "dx", "ddt", "dA", "dB", "dC")] + [
        ("batch", lg), ("L", lg), ("D", lg), ("N", lg),
        ("bc_shared", C.c_int), ("clamp", C.c_int), ("flags", C.c_int), ("pad_", C.c_int)]


class KmbConvND(C.Structure):
    _fields_ = [(n, fp) for n in ("input", "kernel", "bias", "output", "dy", "dinput",
                                  "dkernel", "dbias")] + [
        ("dims", lg * 8), ("ndims", lg), ("batch", lg), ("D", lg), ("K", lg)]


VISIT_FN = C.CFUNCTYPE(C.c_int, C.POINTER(lg), lg, lg, lg, C.c_void_p)

# ---------------------------------------------------------------- kmamba.h
KMAMBA_MAX_NDIMS = 8
OPTIMIZER_ADAM_CLIP, OPTIMIZER_MUON, OPTIMIZER_SGD, OPTIMIZER_ADAMW = 0, 1, 2, 3
_fptr = C.POINTER(C.c_float)


class MBOptimConfig(C.Structure):
    _fields_ = [(n, C.c_float) for n in ("lr", "mu", "beta2", "eps", "clip_norm",
                                         "weight_decay")]


class MBMatrix(C.Structure):
    _fields_ = [("data", _fptr), ("rows", C.c_size_t), ("cols", C.c_size_t)]


class MBConfig(C.Structure):
    _fields_ = [("dim", C.c_size_t), ("state_size", C.c_size_t), ("seq_len", C.c_size_t),
                ("mimo_rank", C.c_size_t), ("dt_scale", C.c_float), ("dt_min", C.c_float),
                ("dt_max", C.c_float), ("use_fp16", C.c_int), ("use_bf16", C.c_int),
                ("loss_scale", C.c_float), ("spatial_ndims", lg),
                ("spatial_dims", lg * KMAMBA_MAX_NDIMS), ("use_convnd", C.c_int),
                ("convnd_K", lg), ("convnd_ndims", lg)]


# parameter tensors of a block in the order of the MBOptimState g_/m_/v_ fields
BLOCK_PARAMS = ("W_in", "W_out", "A_log", "W_B", "W_C", "b_B", "b_C", "delta_proj", "theta",
                "lambda_proj")


class MBOptimState(C.Structure):
    _fields_ = ([("type", C.c_int), ("step", C.c_size_t)]
                + [("g_" + n, _fptr) for n in BLOCK_PARAMS]
                + [(f"{k}_{n}", _fptr) for n in BLOCK_PARAMS for k in ("m", "v")])


class MambaBlockWorkspace(C.Structure):
    _fields_ = [(n, _fptr) for n in ("hidden", "delta", "scan_B", "scan_C", "scan_delta",
                                     "scan_h")]


class MambaBlock(C.Structure):
    _fields_ = [("config", MBConfig), ("W_in", MBMatrix), ("W_out", MBMatrix),
                ("A_log", MBMatrix), ("W_B", MBMatrix), ("W_C", MBMatrix),
                ("delta_proj", MBMatrix), ("b_B", _fptr), ("b_C", _fptr), ("theta", _fptr),
                ("lambda_proj", MBMatrix), ("wavefront_plan", C.c_void_p),
                ("convnd_kernel", _fptr), ("convnd_bias", _fptr), ("hidden", _fptr),
                ("delta", _fptr), ("scan_B", _fptr), ("scan_C", _fptr),
                ("scan_delta", _fptr), ("scan_h", _fptr),
                ("opt_state", C.POINTER(MBOptimState))]


class KMambaConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_size_t), ("dim", C.c_size_t), ("state_size", C.c_size_t),
                ("seq_len", C.c_size_t), ("n_layers", C.c_size_t), ("mimo_rank", C.c_size_t),
                ("dt_scale", C.c_float), ("dt_min", C.c_float), ("dt_max", C.c_float),
                ("spatial_ndims", lg), ("spatial_dims", lg * KMAMBA_MAX_NDIMS),
                ("use_convnd", C.c_int), ("convnd_K", lg), ("convnd_ndims", lg),
                ("weight_tying", C.c_int)]


class KMamba(C.Structure):
    _fields_ = [("cfg", KMambaConfig), ("embedding", _fptr), ("head", _fptr),
                ("layers", C.POINTER(C.POINTER(MambaBlock))), ("for_training", C.c_int),
                ("opt_blocks", MBOptimConfig), ("lr_embed_head", C.c_float),
                ("weight_decay", C.c_float), ("m_embedding", _fptr), ("v_embedding", _fptr),
                ("m_head", _fptr), ("v_head", _fptr), ("step_embed_head", C.c_size_t),
                ("last_grad_norm", C.c_float), ("last_grad_over_clip", C.c_float),
                ("last_grad_would_clip", C.c_int)]


_PB = C.POINTER(MambaBlock)
_PK = C.POINTER(KMamba)
_PW = C.POINTER(MambaBlockWorkspace)
_PS = C.POINTER(MBOptimState)
_PO = C.POINTER(MBOptimConfig)
_PM = C.POINTER(MBMatrix)

MODEL_PROTOTYPES = {
    "mamba_block_create": (_PB, [C.POINTER(MBConfig)]),
    "mamba_block_free": (None, [_PB]),
    "mamba_block_init": (None, [_PB]),
    "mamba_block_workspace_create": (_PW, [_PB]),
    "mamba_block_workspace_free": (None, [_PW]),
    "mamba_block_forward": (None, [_PB, fp, fp, C.c_size_t]),
    "mamba_block_forward_ws": (None, [_PB, _PW, fp, fp, C.c_size_t]),
    "mamba_attach_optimizer": (None, [_PB, C.c_int, _PO]),
    "mamba_free_optimizer": (None, [_PB]),
    "mamba_zero_grads": (None, [_PB]),
    "mamba_optimizer_step": (None, [_PB, _PO]),
    "mamba_block_grad_sqnorm": (C.c_float, [_PB]),
    "mamba_backward": (None, [_PB, fp, fp, fp, C.c_size_t]),
    "mamba_backward_ws": (None, [_PB, _PW, fp, fp, fp, C.c_size_t]),
    "mamba_backward_ws_local": (None, [_PB, _PW, fp, fp, fp, C.c_size_t, _PS]),
    "mamba_local_grad_alloc": (_PS, [_PB]),
    "mamba_local_grad_reduce": (None, [_PB, _PS]),
    "mamba_local_grad_free": (None, [_PS]),
    "mb_matrix_create": (_PM, [C.c_size_t, C.c_size_t]),
    "mb_matrix_free": (None, [_PM]),
    "mb_matrix_zero": (None, [_PM]),
    "mb_matrix_copy": (None, [_PM, _PM]),
    "mb_matrix_vec_mult": (None, [fp, _PM, fp]),
    "mb_vec_add": (None, [fp, fp, C.c_size_t]),
    "mb_vec_scale": (None, [fp, C.c_float, C.c_size_t]),
    "mb_compute_delta": (None, [fp, _PB, fp, C.c_size_t]),
    "kmamba_create": (_PK, [C.POINTER(KMambaConfig)]),
    "kmamba_free": (None, [_PK]),
    "kmamba_init": (C.c_int, [_PK, C.c_uint32]),
    "kmamba_enable_training": (C.c_int, [_PK, _PO, C.c_float, C.c_float]),
    "kmamba_enable_training_with_optimizer": (C.c_int, [_PK, C.c_int, _PO, C.c_float,
                                                        C.c_float]),
    "kmamba_save": (C.c_int, [_PK, C.c_char_p]),
    # device-resident models (kmamba_resident.h)
    "kmamba_set_device_resident": (C.c_int, [_PK, C.c_int]),
    "kmamba_sync_to_host": (C.c_int, [_PK]),
    "kmamba_load": (_PK, [C.c_char_p, C.c_int, _PO, C.c_float, C.c_float]),
    "kmamba_forward": (C.c_int, [_PK, fp, fp]),
    "kmamba_train_step": (C.c_float, [_PK, fp]),
    "kmamba_train_batch": (C.c_float, [_PK, fp, C.c_size_t]),
    "kmamba_train_batch_hybrid": (C.c_float, [_PK, fp, C.c_size_t]),
    "kmamba_last_grad_norm": (C.c_float, [_PK]),
    "kmamba_last_grad_over_clip": (C.c_float, [_PK]),
    "kmamba_last_grad_would_clip": (C.c_int, [_PK]),
    "kmamba_step_count": (C.c_size_t, [_PK]),
    "kmamba_update_lr": (None, [_PK, C.c_float, C.c_float]),
}

# name -> (restype, argtypes)
PROTOTYPES = {
    # runtime
    "kmb_last_error": (C.c_char_p, []),
    "kmb_last_status": (C.c_int, []),
    "kmb_clear_error": (None, []),
    "kmb_set_stream": (None, [C.c_void_p]),
    "kmb_get_stream": (C.c_void_p, []),
    "kmb_set_sync": (None, [C.c_int]),
    "kmb_get_sync": (C.c_int, []),
    "kmb_pool_alloc": (C.c_void_p, [C.c_size_t]),
    "kmb_pool_free": (None, [C.c_void_p]),
    "kmb_pool_trim": (C.c_size_t, []),
    "kmb_pool_bytes_held": (C.c_size_t, []),
    "kmb_block_launch_count": (C.c_ulonglong, []),
    # NCCL data parallelism (kmamba_distributed.h)
    "kmamba_distributed_init_nccl": (C.POINTER(KMambaDistributedContext), [C.c_int, C.c_int]),
    "kmamba_distributed_fini_nccl": (None, [C.POINTER(KMambaDistributedContext)]),
    "kmamba_allreduce_gradients_nccl": (C.c_int, [C.POINTER(KMambaDistributedContext), fp,
                                                  C.c_size_t]),
    "kmamba_broadcast_params_nccl": (C.c_int, [C.POINTER(KMambaDistributedContext), fp,
                                               C.c_size_t]),
    "kmamba_distributed_init_pipeline": (C.POINTER(KMambaDistributedContext), [C.c_int]),
    "kmamba_distributed_fini_pipeline": (None, [C.POINTER(KMambaDistributedContext)]),
    "kmamba_pipeline_send_recv": (C.c_int, [C.POINTER(KMambaDistributedContext), fp, fp,
                                            C.c_size_t, C.c_int, C.c_int]),
    "kmamba_distributed_split_batch": (None, [C.POINTER(KMambaDistributedConfig), C.c_size_t,
                                              C.c_size_t]),
    "kmamba_distributed_split_layers": (None, [C.POINTER(KMambaDistributedConfig),
                                               C.c_size_t, C.c_size_t]),
    "kmb_dist_get_unique_id": (C.c_int, [C.c_void_p]),
    "kmb_dist_init_with_id": (C.POINTER(KMambaDistributedContext), [C.c_int, C.c_int, C.c_int,
                                                                    C.c_void_p]),
    "kmb_dist_rendezvous_file": (C.c_int, [C.c_char_p, C.c_int, C.c_void_p, C.c_size_t,
                                           C.c_double]),
    "kmb_dist_set_bucket_bytes": (C.c_int, [C.POINTER(KMambaDistributedContext), C.c_size_t]),
    "kmb_dist_bucket_add": (C.c_int, [C.POINTER(KMambaDistributedContext), fp, C.c_size_t,
                                      C.c_int, C.c_void_p]),
    "kmb_dist_bucket_flush": (C.c_int, [C.POINTER(KMambaDistributedContext), C.c_void_p]),
    "kmb_dist_wait": (C.c_int, [C.POINTER(KMambaDistributedContext), C.c_void_p]),
    "kmb_dist_stats": (C.c_int, [C.POINTER(KMambaDistributedContext),
                                 C.POINTER(C.c_ulonglong), C.POINTER(C.c_ulonglong)]),
    # Mamba-ND model (kmamba_ndmodel.h)
    "kmb_ndmodel_create": (C.c_void_p, [C.POINTER(KmbNDModelConfig)]),
    "kmb_ndmodel_free": (None, [C.c_void_p]),
    "kmb_ndmodel_param_count": (lg, [C.c_void_p]),
    "kmb_ndmodel_params": (C.c_void_p, [C.c_void_p]),
    "kmb_ndmodel_grads": (C.c_void_p, [C.c_void_p]),
    "kmb_ndmodel_sync_weights": (C.c_int, [C.c_void_p]),
    "kmb_ndmodel_set_dist": (C.c_int, [C.c_void_p, C.POINTER(KMambaDistributedContext)]),
    "kmb_ndmodel_forward": (C.c_int, [C.c_void_p, C.c_void_p, lg, C.POINTER(C.c_float)]),
    "kmb_ndmodel_backward": (C.c_int, [C.c_void_p, C.c_void_p, lg, C.POINTER(C.c_float)]),
    "kmb_ndmodel_step": (C.c_int, [C.c_void_p, C.c_float, C.c_float]),
    "kmb_ndmodel_train_step": (C.c_int, [C.c_void_p, C.c_void_p, lg, C.c_float, C.c_float,
                                         C.POINTER(C.c_float)]),
    # tensor-core GEMM
    "kmb_gemm_bf16": (C.c_int, [C.POINTER(KmbGemm)]),
    "kmb_gemm_check_error": (C.c_int, []),
    # 1D scan
    "kmb_scan1d_ckpt_elems": (lg, [lg, lg, lg, lg]),
    # segments and steps per segment the 1D entry points split L into
    "kmb_scan1d_seg_plan": (C.c_int, [lg, lg, lg, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    # diagnostic: the FMA-pipe 2^w of the scans on device pointers
    "kmb_exp2_fma_eval": (C.c_int, [C.c_void_p, C.c_void_p, lg]),
    "kmb_scan1d_fwd": (C.c_int, [C.POINTER(KmbScan1D)]),
    "kmb_scan1d_bwd": (C.c_int, [C.POINTER(KmbScan1D)]),
    "kmb_scan1d_bwd_noalloc": (C.c_int, [C.POINTER(KmbScan1D)]),
    "kmb_scan1d_fwd_bf16": (C.c_int, [C.POINTER(KmbScan1D)]),
    "kmb_scan1d_bwd_bf16": (C.c_int, [C.POINTER(KmbScan1D)]),
    "scan1d": (None, [C.POINTER(ScanParams)]),
    "scan1d_backward": (None, [C.POINTER(ScanBackwardParams)]),
    "scan1d_backward_m1_shared_bc": (None, [C.POINTER(ScanBackwardSharedParams)]),
    "scan1d_backward_m1_shared_bc_asm": (None, [C.POINTER(ScanBackwardSharedParams)]),
    "scan1d_backward_m1_shared_bc_simple_asm": (None, [C.POINTER(ScanBackwardSharedParams)]),
    "om_scan1d_forward": (None, [fp] * 7 + [C.c_int] * 3),
    "om_scan1d_backward": (None, [fp] * 12 + [C.c_int] * 3),
    "mamba_scan1d_forward": (None, [C.POINTER(ScanParams)]),
    "mamba_scan1d_backward": (None, [C.POINTER(ScanBackwardParams)]),
    "mamba_scan1d_backward_m1_shared_bc": (None, [C.POINTER(ScanBackwardSharedParams)]),
    "mamba_scan1d_cuda_forward": (None, [fp] * 7 + [C.c_int] * 3),
    "mamba_scan1d_cuda_backward": (None, [fp] * 12 + [C.c_int] * 3),
    # ConvND
    "convnd_kernel_volume": (lg, [lg, lg]),
    "convnd": (None, [C.POINTER(ConvNDParams), C.c_int]),
    "convnd_forward_wavefront": (None, [C.POINTER(ConvNDParams), C.POINTER(KMWavefrontPlan)]),
    "convnd_backward_wavefront": (None, [C.POINTER(ConvNDParams), C.POINTER(KMWavefrontPlan)]),
    "om_convnd_forward": (C.c_int, [C.POINTER(ConvNDParams)]),
    "om_convnd_backward": (C.c_int, [C.POINTER(ConvNDParams)]),
    "kmb_convnd_fwd": (C.c_int, [C.POINTER(KmbConvND)]),
    "kmb_convnd_bwd": (C.c_int, [C.POINTER(KmbConvND)]),
    "kmb_convnd_fwd_bf16": (C.c_int, [C.POINTER(KmbConvND)]),
    "kmb_convnd_bwd_bf16": (C.c_int, [C.POINTER(KmbConvND)]),
    # topology
    "wavefront_nd_validate_dims": (C.c_int, [fp, lg]),
    "wavefront_nd_total_points": (lg, [fp, lg]),
    "wavefront_nd_max_level": (lg, [fp, lg]),
    "wavefront_nd_row_major_offset": (lg, [fp, fp, lg]),
    "wavefront_nd_level_size": (lg, [fp, lg, lg]),
    "wavefront_nd_for_level": (C.c_int, [fp, lg, lg, fp, VISIT_FN, C.c_void_p]),
    "wavefront_nd_for_each_level": (C.c_int, [fp, lg, fp, VISIT_FN, C.c_void_p]),
    "km_wavefront_plan_create": (C.POINTER(KMWavefrontPlan), [fp, lg]),
    "km_wavefront_plan_free": (None, [C.POINTER(KMWavefrontPlan)]),
    "km_wavefront_plan_matches_dims": (C.c_int, [C.POINTER(KMWavefrontPlan), fp, lg]),
    "km_wavefront_plan_level_size": (lg, [C.POINTER(KMWavefrontPlan), lg]),
    "km_wavefront_plan_level_offsets": (C.POINTER(lg), [C.POINTER(KMWavefrontPlan), lg]),
    "km_spatial_dims_product": (C.c_int, [fp, lg, C.POINTER(C.c_size_t)]),
    "km_make_row_major_strides": (C.c_int, [fp, lg, fp]),
    "km_unravel_index": (None, [lg, fp, fp, lg, fp]),
    "km_ravel_index": (lg, [fp, fp, fp, lg]),
    "km_power_long": (lg, [lg, lg]),
    "km_normalize_spatial_topology": (C.c_int, [fp, fp, C.c_size_t, C.c_int, fp, lg]),
    # km_memory_pool.h over device memory
    "km_memory_pool_create": (C.c_void_p, []),
    "km_memory_pool_destroy": (None, [C.c_void_p]),
    "km_pool_alloc": (C.c_void_p, [C.c_void_p, C.c_size_t]),
    "km_pool_free": (None, [C.c_void_p, C.c_void_p]),
    "km_pool_clear": (None, [C.c_void_p]),
    "km_memory_pool_threadlocal": (C.c_void_p, []),
    "km_memory_pool_destroy_all_threadlocal": (None, []),
}


def load(path: str = LIB_PATH):
    """Loads the library and declares every prototype.  Raises OSError when
    the library is missing (the product has no fallback)."""
    lib = C.CDLL(path)
    declare(lib)
    return lib


def declare(lib, table=None):
    """Sets restype/argtypes of every known prototype present in `lib`
    (also used for the reference library the tests load as the oracle)."""
    for name, (res, args) in (table or {**PROTOTYPES, **MODEL_PROTOTYPES}).items():
        f = getattr(lib, name, None)
        if f is None:
            continue
        f.restype = res
        f.argtypes = args


def last_error(lib) -> str:
    s = lib.kmb_last_error()
    return s.decode() if s else ""


def check(lib, status: int) -> None:
    if status != KMB_OK:
        raise RuntimeError(f"kmamba_b200 status {status}: {last_error(lib)}")


def as_array(ptr, n):
    """numpy view of n floats at a float* field (host memory)."""
    import numpy as np
    return np.ctypeslib.as_array(ptr, shape=(int(n),))


def block_tensor(block, name):
    """numpy view of one parameter of a MambaBlock (host arrays)."""
    b = block.contents if hasattr(block, "contents") else block
    c = b.config
    R = max(int(c.mimo_rank), 1)
    N, D = int(c.state_size), int(c.dim)
    sizes = {"W_in": R * D, "W_out": D * R, "A_log": N, "W_B": N * R * D, "W_C": N * R * D,
             "b_B": N * R, "b_C": N * R, "delta_proj": D, "lambda_proj": D,
             "theta": max(N // 2, 1)}
    f = getattr(b, name)
    return as_array(f.data if isinstance(f, MBMatrix) else f, sizes[name])


def block_state(block, prefix, name):
    """numpy view of g_/m_/v_<name> of a block's optimizer state."""
    b = block.contents if hasattr(block, "contents") else block
    n = block_tensor(b, name).size
    return as_array(getattr(b.opt_state.contents, f"{prefix}_{name}"), n)
