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
    # 1D scan
    "kmb_scan1d_ckpt_elems": (lg, [lg, lg, lg, lg]),
    "kmb_scan1d_fwd": (C.c_int, [C.POINTER(KmbScan1D)]),
    "kmb_scan1d_bwd": (C.c_int, [C.POINTER(KmbScan1D)]),
    "kmb_scan1d_bwd_noalloc": (C.c_int, [C.POINTER(KmbScan1D)]),
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
}


def load(path: str = LIB_PATH):
    """Loads the library and declares every prototype.  Raises OSError when
    the library is missing (the product has no fallback)."""
    lib = C.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        f = getattr(lib, name, None)
        if f is None:
            continue
        f.restype = res
        f.argtypes = args
    return lib


def last_error(lib) -> str:
    s = lib.kmb_last_error()
    return s.decode() if s else ""


def check(lib, status: int) -> None:
    if status != KMB_OK:
        raise RuntimeError(f"kmamba_b200 status {status}: {last_error(lib)}")
