"""ctypes binding of ``libparrot_b200.so`` (the C ABI in ``include/parrot_b200.h``).

There is no fallback: if the library is missing or the device is not an
sm_100 GPU, calls raise ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libparrot_b200.so")

PARROT_OK = 0
PARROT_EINVAL = -1
PARROT_ECUDA = -2


class MoeDims(ctypes.Structure):
    _fields_ = [("tokens", c_int), ("dim", c_int), ("n_experts", c_int), ("top_k", c_int),
                ("expert_dim", c_int), ("shared_dim", c_int), ("capacity", c_int)]


class MoeWeights(ctypes.Structure):
    _fields_ = [("router", c_void_p), ("router_bias", c_void_p), ("gate_up", c_void_p),
                ("down", c_void_p), ("shared_gate_up", c_void_p), ("shared_down", c_void_p)]


class MoeOutputs(ctypes.Structure):
    _fields_ = [("out", c_void_p), ("residual", c_void_p), ("probs", c_void_p),
                ("indices", c_void_p), ("weights", c_void_p), ("positions", c_void_p),
                ("counts", c_void_p), ("stats", c_void_p)]


LAYOUT_OFFSETS = ("indices", "weights", "positions", "chunk_hist", "tile_hist",
                  "tile_probsum", "counts", "seg_rows", "seg_base", "stats",
                  "status", "row_dst", "row_w", "grouped", "hidden", "contrib",
                  "shared_hidden", "shared_y", "total")


class MoeLayout(ctypes.Structure):
    _fields_ = [(name, c_size_t) for name in LAYOUT_OFFSETS] + [
        ("capacity", c_int), ("grouped_rows", c_int), ("route_blocks", c_int),
        ("reserved", c_int)]


EP_MAX_RANKS = 8


class EpDims(ctypes.Structure):
    _fields_ = [("ranks", c_int), ("rank", c_int), ("max_tokens", c_int), ("dim", c_int),
                ("n_experts", c_int), ("expert_dim", c_int), ("wait_ns", ctypes.c_ulonglong),
                ("slots", c_int), ("plan", (ctypes.c_byte * 32) * EP_MAX_RANKS)]


EP_LAYOUT_OFFSETS = ("flags_in", "flags_back", "meta", "recv_rows", "back_rows", "epoch",
                     "counters", "status", "seg_rows", "seg_base", "seg_expert", "back_n",
                     "back_base", "hidden", "y", "total")


class EpLayout(ctypes.Structure):
    _fields_ = [(name, c_size_t) for name in EP_LAYOUT_OFFSETS] + [
        ("region_rows", c_int), ("reserved", c_int)]


class EpPeers(ctypes.Structure):
    _fields_ = [("buffers", c_void_p * EP_MAX_RANKS)]


_SIGNATURES = {
    "parrot_b200_version": (c_int, []),
    "parrot_b200_last_error": (ctypes.c_char_p, []),
    "parrot_b200_device_supported": (c_int, [c_int]),
    "parrot_rmsnorm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "parrot_depthmix_bf16": (c_int, [c_void_p, POINTER(c_void_p), c_int, c_void_p, c_void_p,
                                     c_float, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_int, c_int, c_void_p]),
    "parrot_depthmix_moe_bf16": (c_int, [c_void_p, POINTER(c_void_p), c_int, c_void_p, c_void_p,
                                         c_float, c_void_p, c_float, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "parrot_rope_inplace_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_int, c_int, c_int, c_int, c_void_p]),
    "parrot_rope_inplace_at_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                            c_int, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "parrot_decode_attention_bf16": (c_int, [c_void_p, c_int, c_void_p, c_int,
                                             ctypes.c_longlong, c_void_p, c_void_p,
                                             ctypes.c_longlong, c_void_p, c_void_p, c_void_p,
                                             c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                             c_void_p, c_size_t, c_void_p, c_void_p]),
    "parrot_decode_attention_rope_bf16": (c_int, [c_void_p, c_int, c_void_p, ctypes.c_longlong,
                                                  c_void_p, c_void_p, ctypes.c_longlong, c_void_p,
                                                  c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                                  c_int, c_int, c_float, c_void_p, c_void_p,
                                                  c_int, c_void_p, c_size_t, c_void_p, c_void_p]),
    "parrot_linear_small": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
                                    c_int, c_int, c_void_p]),
    "parrot_decode_attention_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "parrot_moe_capacity": (c_int, [c_int, c_int]),
    "parrot_moe_workspace_layout": (c_int, [POINTER(MoeDims), POINTER(MoeLayout)]),
    "parrot_moe_workspace_init": (c_int, [c_void_p, POINTER(MoeDims), c_void_p]),
    "parrot_pack_gate_up_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_void_p]),
    "parrot_pack_down_bf16": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "parrot_silu_bf16": (c_int, [c_void_p, c_void_p, ctypes.c_int64, c_void_p]),
    "parrot_moe_forward_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                        POINTER(MoeOutputs), c_void_p, c_size_t, c_void_p]),
    "parrot_moe_forward_deferred_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                                 POINTER(MoeOutputs), c_void_p, c_size_t,
                                                 c_void_p]),
    "parrot_moe_forward_static_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                               POINTER(MoeOutputs), c_void_p]),
    "parrot_depthmix_route_bf16": (c_int, [c_void_p, POINTER(c_void_p), c_int, c_void_p,
                                           c_void_p, c_float, c_void_p, c_float, c_void_p,
                                           c_void_p, c_void_p, c_void_p, c_int, c_int,
                                           POINTER(MoeDims), POINTER(MoeWeights),
                                           POINTER(MoeOutputs), c_void_p, c_size_t, c_void_p]),
    "parrot_moe_forward_routed_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                               POINTER(MoeOutputs), c_int, c_void_p, c_size_t,
                                               c_void_p]),
    "parrot_moe_decode_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                       POINTER(MoeOutputs), c_void_p, c_size_t, c_void_p]),
    "parrot_moe_decode_routed_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                       POINTER(MoeOutputs), c_void_p, c_size_t, c_void_p]),
    "parrot_moe_route_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                      POINTER(MoeOutputs), c_void_p, c_size_t, c_void_p]),
    "parrot_moe_experts_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                        POINTER(MoeOutputs), c_void_p, c_size_t, c_void_p]),
    "parrot_moe_gemm_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p, c_void_p,
                                     c_size_t, c_int, c_void_p]),
    "parrot_b200_launch_count": (ctypes.c_ulonglong, []),
    "parrot_moe_read_status": (c_int, [c_void_p, POINTER(MoeDims), POINTER(c_int), c_void_p]),
    "parrot_moe_ep_dispatch_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                            POINTER(MoeOutputs), c_int, c_void_p, c_size_t,
                                            c_void_p]),
    "parrot_moe_shared_ffn_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights), c_void_p,
                                           c_void_p, c_size_t, c_void_p]),
    "parrot_moe_expert_ffn_bf16": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_void_p]),
    "parrot_moe_ep_combine_bf16": (c_int, [POINTER(MoeDims), c_void_p, c_void_p, c_size_t,
                                           c_void_p, c_void_p, c_void_p]),
    "parrot_vocab_argmax_scratch_bytes": (c_size_t, []),
    "parrot_vocab_argmax_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_void_p, c_size_t, c_void_p]),
    "parrot_argmax_rows_bf16": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "parrot_ep_buffer_layout": (c_int, [POINTER(EpDims), POINTER(EpLayout)]),
    "parrot_ipc_export": (c_int, [c_void_p, c_void_p, POINTER(ctypes.c_ulonglong)]),
    "parrot_ipc_import": (c_int, [c_void_p, ctypes.c_ulonglong, POINTER(c_void_p),
                                  POINTER(c_void_p)]),
    "parrot_ipc_close": (c_int, [c_void_p]),
    "parrot_moe_ep_dispatch_planned_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights),
                                                    c_void_p, POINTER(MoeOutputs),
                                                    POINTER(EpDims), c_void_p, c_size_t,
                                                    c_void_p]),
    "parrot_moe_ep_send_bf16": (c_int, [POINTER(MoeDims), POINTER(EpDims), POINTER(EpPeers),
                                        c_void_p, c_size_t, c_void_p]),
    "parrot_moe_ep_receive": (c_int, [POINTER(EpDims), c_void_p, c_void_p]),
    "parrot_moe_ep_experts_bf16": (c_int, [POINTER(EpDims), c_void_p, c_void_p, c_void_p,
                                           c_void_p]),
    "parrot_moe_ep_return_bf16": (c_int, [POINTER(EpDims), POINTER(EpPeers), c_void_p]),
    "parrot_moe_ep_dispatch_send_bf16": (c_int, [POINTER(MoeDims), POINTER(MoeWeights),
                                                 c_void_p, POINTER(MoeOutputs), POINTER(EpDims),
                                                 POINTER(EpPeers), c_void_p, c_size_t,
                                                 c_void_p]),
    "parrot_moe_ep_experts_return_bf16": (c_int, [POINTER(EpDims), POINTER(EpPeers), c_void_p,
                                                  c_void_p, c_void_p]),
    "parrot_moe_ep_combine_peer_bf16": (c_int, [POINTER(MoeDims), POINTER(EpDims), c_void_p,
                                                c_void_p, c_size_t, c_void_p, c_void_p,
                                                c_void_p]),
    "parrot_ep_read_status": (c_int, [POINTER(EpDims), c_void_p, POINTER(c_int), c_void_p]),
    "parrot_selftest_wait_timeout": (c_int, [ctypes.c_ulonglong, c_void_p, c_void_p]),
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (once) and declare every entry point's signature."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m parrot_b200.build` "
                "(nvcc 12.9, sm_100a). The B200 backend has no fallback.")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def check(rc: int, what: str) -> None:
    """Turn a non-zero C status into ``RuntimeError`` naming the kernel."""
    if rc != PARROT_OK:
        msg = load().parrot_b200_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def exported_names() -> list[str]:
    return list(_SIGNATURES)
