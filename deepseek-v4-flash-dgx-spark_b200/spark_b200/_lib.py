"""ctypes binding of libdsv4moe.so (the C ABI declared in include/dsv4moe.h).

Every call returns a status code; non-zero codes become ``RuntimeError`` with
the message the reference's ``TORCH_CHECK`` would raise
(spark_runtime/native/native_packed_loader.cpp:27-33,77-108,128-160,203-207,265,299).
There is no fallback: if the library cannot be loaded, importing a module that
needs it raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "lib" / "libdsv4moe.so"

c_int = ctypes.c_int
c_ll = ctypes.c_longlong
c_float = ctypes.c_float
c_double = ctypes.c_double
c_vp = ctypes.c_void_p
c_ip = ctypes.POINTER(ctypes.c_int)
c_llp = ctypes.POINTER(ctypes.c_longlong)
c_dp = ctypes.POINTER(ctypes.c_double)

OK = 0
ERR_ARG = -1
ERR_CUDA = -2
ERR_UNSUPPORTED = -3
ERR_IO = -4
ERR_SHORT_READ = -5
ERR_BOUNDS = -6
ERR_SIZE = -7
ERR_WORKSPACE = -8

DEVERR_NAMES = {
    101: "TMA producer wait timed out",
    102: "MMA issuer wait timed out",
    103: "epilogue wait timed out",
    104: "expert index out of range",
    105: "routing plan exceeds its workspace",
    106: "materializer source offset not 16-byte aligned",
    107: "a peer rank's exchange flag did not arrive in time",
}


class MoELayerDesc(ctypes.Structure):
    """Mirror of ``struct dsv4_moe_layer``."""

    _fields_ = [
        ("hidden", c_int),
        ("inter", c_int),
        ("n_routed", c_int),
        ("topk", c_int),
        ("n_shared", c_int),
        ("route_scale", c_float),
        ("swiglu_limit", c_float),
        ("gate_w", c_vp),
        ("gate_w_fp32", c_int),
        ("gate_bias", c_vp),
        ("arena", c_vp),
        ("slot_stride", c_ll),
        ("n_slots", c_int),
        ("arena_sf", c_vp),
        ("sf_slot_stride", c_ll),
        ("expert_slot", c_vp),
        ("shared_w1", c_vp),
        ("shared_w2", c_vp),
        ("shared_w3", c_vp),
        ("shared_sf", c_vp),
    ]


_SIGNATURES = {
    "dsv4_version": (c_int, []),
    "dsv4_kernel_launches": (c_ll, []),
    "dsv4_status_string": (ctypes.c_char_p, [c_int]),
    "dsv4_device_error": (c_int, [c_int, c_ip]),
    "dsv4_device_error_async": (c_int, [c_vp, c_vp]),
    "dsv4_set_k_split": (c_int, [c_int]),
    "dsv4_set_fp4_activations": (c_int, [c_int]),
    "dsv4_settings_generation": (c_ll, []),
    "dsv4_set_fused_routing": (c_int, [c_int]),
    "dsv4_fp4_act_quant": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "dsv4_fp8_weight_atoms_bytes": (c_ll, [c_int, c_int]),
    "dsv4_build_fp8_weight_atoms": (c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    "dsv4_fp8_linear_workspace_bytes": (c_ll, [c_int, c_int, c_int]),
    "dsv4_fp8_linear": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_int, c_vp, c_vp, c_ll, c_vp]),
    "dsv4_sparse_attn_workspace_bytes": (c_ll, [c_int, c_int, c_int]),
    "dsv4_sparse_attn": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                 c_vp, c_vp, c_ll, c_vp]),
    "dsv4_moe_workspace_bytes": (c_ll, [ctypes.POINTER(MoELayerDesc), c_int]),
    "dsv4_moe_workspace_layout": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_llp, c_int]),
    "dsv4_moe_forward": (c_int, [ctypes.POINTER(MoELayerDesc), c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_ll, c_vp]),
    "dsv4_expert_workspace_bytes": (c_ll, [ctypes.POINTER(MoELayerDesc), c_int]),
    "dsv4_expert_forward": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_ll, c_vp]),
    "dsv4_expert_static_scratch_bytes": (c_ll, []),
    "dsv4_expert_forward_static": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_vp, c_int, c_vp, c_vp, c_vp]),
    "dsv4_profile_enable": (c_int, [c_int]),
    "dsv4_profile_read": (c_int, [ctypes.POINTER(c_float), c_int]),
    "dsv4_gate_logits": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "dsv4_gate_workspace_bytes": (c_ll, [c_vp, c_int, c_int, c_int, c_int]),
    "dsv4_gate_route": (c_int, [c_vp, c_vp, c_int, c_vp, c_int, c_int, c_int, c_int, c_float, c_vp, c_vp, c_vp,
                                c_vp, c_ll, c_vp]),
    "dsv4_gate_topk": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_float, c_vp, c_vp, c_vp]),
    "dsv4_act_quant": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "dsv4_materialize": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_ll, c_vp, c_ll, c_vp, c_ll, c_vp]),
    "dsv4_build_scale_atoms": (c_int, [c_vp, c_ll, c_vp, c_int, c_int, c_int, c_vp, c_ll, c_vp]),
    "dsv4_build_shared_scale_atoms": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    "dsv4_read_into": (c_int, [c_int, c_vp, c_ll, c_ll, c_ll, c_llp, c_ip]),
    "dsv4_copy_slices": (c_int, [c_vp, c_ll, ctypes.POINTER(c_vp), c_llp, c_llp, c_llp, c_int, c_int, c_vp, c_llp]),
    "dsv4_read_into_and_copy": (
        c_int,
        [c_int, c_vp, c_ll, c_ll, c_ll, ctypes.POINTER(c_vp), c_llp, c_llp, c_llp, c_int, c_int, c_vp,
         c_llp, c_llp, c_dp, c_dp, c_ip],
    ),
    "dsv4_gate_hash_workspace_bytes": (c_ll, [c_vp, c_int, c_int, c_int, c_int]),
    "dsv4_gate_route_hash": (c_int, [c_vp, c_vp, c_int, c_vp, c_ll, c_vp, c_int, c_int, c_int, c_int, c_float,
                                     c_vp, c_vp, c_vp, c_vp, c_ll, c_vp]),
    "dsv4_ep_row_bytes": (c_ll, [c_int, c_int]),
    "dsv4_ep_dispatch_workspace_bytes": (c_ll, [c_int, c_int]),
    "dsv4_ep_dispatch": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_ll, c_vp, c_vp,
                                 c_vp, c_ll, c_vp]),
    "dsv4_ep_expert_workspace_bytes": (c_ll, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_int]),
    "dsv4_ep_expert_forward": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_vp, c_int, c_vp, c_int,
                                       c_vp, c_vp, c_ll, c_vp, c_ll, c_vp]),
    "dsv4_ep_combine": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_vp, c_vp, c_vp, c_int, c_int,
                                c_vp, c_ll, c_vp, c_vp]),
    "dsv4_ep_exchange_bytes": (c_ll, [c_int, c_int, c_int, c_int]),
    "dsv4_ep_exchange_alloc": (c_int, [c_int, c_ll, ctypes.POINTER(c_vp)]),
    "dsv4_ep_exchange_free": (c_int, [c_vp]),
    "dsv4_ipc_handle": (c_int, [c_vp, c_vp]),
    "dsv4_ipc_open": (c_int, [c_int, c_vp, ctypes.POINTER(c_vp)]),
    "dsv4_ipc_close": (c_int, [c_vp]),
    "dsv4_ep_p2p_dispatch_workspace_bytes": (c_ll, [c_int, c_int]),
    "dsv4_ep_dispatch_p2p": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_int,
                                     c_int, c_vp, c_vp, c_ll, c_vp]),
    "dsv4_ep_p2p_expert_workspace_bytes": (c_ll, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_int]),
    "dsv4_ep_expert_forward_p2p": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_vp, c_int, c_vp, c_vp,
                                           c_int, c_int, c_vp, c_ll, c_vp]),
    "dsv4_ep_combine_p2p": (c_int, [ctypes.POINTER(MoELayerDesc), c_int, c_int, c_vp, c_vp, c_vp, c_int, c_int,
                                    c_int, c_vp, c_ll, c_vp, c_vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def load(path: Path | str | None = None):
    """Load (once) and return the ctypes handle; raises if the library is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else Path(os.environ.get("DSV4MOE_LIB", LIB_PATH))
    if not p.exists():
        raise RuntimeError(
            f"libdsv4moe.so not found at {p}; build it with "
            "`python deepseek-v4-flash-dgx-spark_b200/build.py` (there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


_MESSAGES = {
    ERR_ARG: "invalid argument",
    ERR_CUDA: "CUDA error",
    ERR_UNSUPPORTED: "unsupported shape or option",
    ERR_IO: "pread failed",
    ERR_SHORT_READ: "short packed expert read",
    ERR_BOUNDS: "source slice exceeds storage tensor",
    ERR_SIZE: "target size does not match expert copy plan",
    ERR_WORKSPACE: "workspace too small",
}


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = _MESSAGES.get(status, f"status {status}")
    raise RuntimeError(f"{what}: {msg}" if what else msg)


def device_error(clear: bool = True) -> int:
    code = c_int(0)
    check(load().dsv4_device_error(1 if clear else 0, ctypes.byref(code)), "dsv4_device_error")
    return code.value


def raise_on_device_error() -> None:
    code = device_error(clear=True)
    if code:
        raise RuntimeError(f"device-side error {code}: {DEVERR_NAMES.get(code, 'unknown')}")


def ptr(t) -> int:
    """Data pointer of a torch tensor (0 for None)."""
    return 0 if t is None else int(t.data_ptr())


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)
