"""Loader for libvdxsampler.so with ctypes signatures for every entry point of
include/vdx_sampler.h. Importing this module never touches a GPU."""
from __future__ import annotations

import ctypes as C
import os

from .abi import VdxsConfig

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvdxsampler.so")

_lib = None

P = C.POINTER
vp = C.c_void_p
i32 = C.c_int32
i64 = C.c_int64

# name -> (restype, argtypes); mirrors include/vdx_sampler.h
SIGNATURES = {
    "vdxs_abi_version": (i32, []),
    "vdxs_default_config": (None, [P(VdxsConfig)]),
    "vdxs_create": (i32, [i32, P(vp)]),
    "vdxs_destroy": (i32, [vp]),
    "vdxs_last_error": (C.c_char_p, [vp]),
    "vdxs_set_tie_mode": (i32, [vp, i32]),
    "vdxs_get_tie_mode": (i32, [vp, P(i32)]),
    "vdxs_sample": (i32, [vp, P(VdxsConfig), vp, i32, i32, i32, i64, vp, i64, vp, vp, vp, vp]),
    "vdxs_sample_ex": (i32, [vp, P(VdxsConfig), vp, i32, i32, i32, i64, vp, i64, vp, vp, vp, vp, vp,
                             vp, i32, vp]),
    "vdxs_sample_host": (i32, [vp, P(VdxsConfig), vp, i32, i32, i32, i64, vp, i64, vp, vp, vp, vp]),
    "vdxs_sample_noalloc": (i32, [P(VdxsConfig), i32, vp, i32, i32, i32, i64, vp, i64, vp, vp, vp, vp]),
    "vdxs_noalloc_status": (i32, [vp]),
    "vdxs_device_uniforms": (i32, [vp, i32, vp, vp]),
    "vdxs_device_history_push": (i32, [vp, vp, vp, i32, vp, i32, vp, i32, vp, vp]),
    "vdxs_decode_step": (i32, [vp, P(VdxsConfig), vp, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, i32, vp, vp, vp]),
    "vdxs_sampler_create": (i32, [vp, i32, P(vp)]),
    "vdxs_sampler_destroy": (i32, [vp]),
    "vdxs_sampler_set_config": (i32, [vp, P(VdxsConfig)]),
    "vdxs_sampler_get_config": (i32, [vp, P(VdxsConfig)]),
    "vdxs_sampler_add_to_history": (i32, [vp, i32, i32]),
    "vdxs_sampler_add_to_history_batch": (i32, [vp, vp]),
    "vdxs_sampler_reset_history": (i32, [vp, i32]),
    "vdxs_sampler_process": (i32, [vp, vp, i32, i32, i64, vp, vp]),
    "vdxs_sampler_process_host": (i32, [vp, vp, i32, i64, vp]),
    "vdxs_sampler_next_float": (i32, [vp, i32, P(C.c_float)]),
    "vdxs_sampler_get_prng_state": (i32, [vp, i32, P(C.c_uint64)]),
    "vdxs_sampler_set_prng_state": (i32, [vp, i32, P(C.c_uint64)]),
    "vdxs_sampler_get_history": (i32, [vp, i32, vp, i32, P(i32), P(i32)]),
    "vdxs_comm_unique_id": (i32, [vp]),
    "vdxs_comm_create": (i32, [vp, i32, i32, vp, P(vp)]),
    "vdxs_comm_create_ex": (i32, [vp, i32, i32, vp, i32, P(vp)]),
    "vdxs_comm_abort": (i32, [vp]),
    "vdxs_comm_status": (i32, [vp]),
    "vdxs_comm_wait": (i32, [vp, vp, i32]),
    "vdxs_comm_destroy": (i32, [vp]),
    "vdxs_sample_sharded": (i32, [vp, vp, P(VdxsConfig), vp, i32, i32, i32, i64, i64, i64, vp, i64, vp,
                                  vp, vp, vp, vp]),
    "vdxs_device_status": (i32, [vp, vp]),
    "vdxs_set_stage_events": (i32, [vp, vp, vp]),
    "vdxs_get_launch_count": (i32, [vp, P(i64)]),
    "vdxs_q4_0_prepare": (i32, [vp, vp, i32, i32, vp, P(vp)]),
    "vdxs_q4_0_release": (i32, [vp]),
    "vdxs_unembed_q4_0": (i32, [vp, vp, vp, i32, vp, vp]),
    "vdxs_sample_unembed_q4_0": (i32, [vp, P(VdxsConfig), vp, vp, i32, vp, i64, vp, vp, vp, vp]),
}


class VdxsError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"vdxs error {code}: {message}")
        self.code = code


def load(path: str | None = None):
    """Load the library (once). Raises if the built .so is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing; build it with `python -m vindexllm_b200.build`")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.vdxs_abi_version() != 1:
        raise ImportError("libvdxsampler.so ABI version mismatch")
    _lib = lib
    return lib


def check(rc: int, ctx=None):
    if rc != 0:
        msg = load().vdxs_last_error(ctx)
        raise VdxsError(rc, (msg or b"").decode(errors="replace"))
