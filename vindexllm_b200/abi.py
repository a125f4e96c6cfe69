"""ctypes mirror of include/vdx_sampler.h: the config record, codes and flags.

``VdxsConfig`` mirrors TVdxSamplerConfig (src/VindexLLM.Sampler.pas:26-34) under the
reference's {$A8} alignment (src/VindexLLM.Defines.inc:13): 32 bytes, seed at 24.
"""
from __future__ import annotations

import ctypes as C

ABI_VERSION = 1

OK = 0
E_INVALID_ARG = -1
E_CUDA = -2
E_NCCL = -3
E_TIMEOUT = -4
E_UNSUPPORTED = -5
E_NO_MEMORY = -6
E_DEVICE_STATE = -7

DTYPE_F32 = 0
DTYPE_BF16 = 1

TIES_FAITHFUL = 0
TIES_CANONICAL = 1

FLAG_GREEDY = 1 << 0
FLAG_TOPK = 1 << 1
FLAG_FULL = 1 << 2
FLAG_BOUNDARY_TIE = 1 << 3
FLAG_DRAW_TIE_RUN = 1 << 4
FLAG_NEAR_BOUNDARY = 1 << 5
FLAG_INEXACT_SUM = 1 << 6
FLAG_FALLBACK = 1 << 7
FLAG_SLOT_ORDER = 1 << 8
FLAG_FAITHFUL_PASS = 1 << 9

FLAG_NAMES = {
    FLAG_GREEDY: "greedy", FLAG_TOPK: "topk", FLAG_FULL: "full",
    FLAG_BOUNDARY_TIE: "boundary_tie", FLAG_DRAW_TIE_RUN: "draw_tie_run",
    FLAG_NEAR_BOUNDARY: "near_boundary", FLAG_INEXACT_SUM: "inexact_sum",
    FLAG_FALLBACK: "fallback", FLAG_SLOT_ORDER: "slot_order",
    FLAG_FAITHFUL_PASS: "faithful_pass",
}


class VdxsConfig(C.Structure):
    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_int32),
        ("top_p", C.c_float),
        ("min_p", C.c_float),
        ("repeat_penalty", C.c_float),
        ("repeat_window", C.c_int32),
        ("seed", C.c_int64),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}

    @classmethod
    def from_dict(cls, d: dict) -> "VdxsConfig":
        c = cls()
        for name, _ in cls._fields_:
            setattr(c, name, d[name])
        return c

    def __repr__(self) -> str:
        return f"VdxsConfig({self.as_dict()})"


assert C.sizeof(VdxsConfig) == 32 and VdxsConfig.seed.offset == 24


def default_config(**overrides) -> VdxsConfig:
    """TVdxSampler.DefaultConfig (Sampler.pas:100-109), with optional overrides."""
    d = dict(temperature=0.0, top_k=0, top_p=1.0, min_p=0.0, repeat_penalty=1.0,
             repeat_window=64, seed=0)
    d.update(overrides)
    return VdxsConfig.from_dict(d)
