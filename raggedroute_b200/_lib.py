"""ctypes loader and signatures for libraggedroute_b200.so (the C ABI in
include/raggedroute_b200.h). Loading fails loudly: there is no fallback."""
from __future__ import annotations

import ctypes
import dataclasses
import enum
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
library_path = os.path.join(_PKG, "libraggedroute_b200.so")

MAX_EXPERTS = 1024
ARCH_AUTO, ARCH_SM86, ARCH_SM90, ARCH_OTHER, ARCH_SM100 = 0, 1, 2, 3, 4
FAMILY_AUTO, FAMILY_CUDA_NAIVE, FAMILY_CUDA_OPTIMIZED = 0, 1, 2


class StatusCode(enum.IntEnum):
    """Equal to raggedroute::StatusCode (include/raggedroute/status.h:7-16),
    plus COMM_ERROR for the expert-parallel runtime."""
    SUCCESS = 0
    INVALID_ARGUMENT = 1
    UNSUPPORTED_ARCHITECTURE = 2
    UNSUPPORTED_DATA_TYPE = 3
    UNSUPPORTED_LAYOUT = 4
    UNSUPPORTED_KERNEL_VARIANT = 5
    INSUFFICIENT_WORKSPACE = 6
    CUDA_ERROR = 7
    COMM_ERROR = 8


class RaggedRouteError(RuntimeError):
    def __init__(self, code: int, cuda_error: int, message: str, op: str):
        self.code = StatusCode(code)
        self.cuda_error = cuda_error
        self.message = message
        super().__init__(f"{op}: {self.code.name}: {message}"
                         + (f" (cudaError {cuda_error})" if cuda_error else ""))


class RRStatus(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("cuda_error", ctypes.c_int32),
                ("message", ctypes.c_char_p)]


class RRContext(ctypes.Structure):
    _fields_ = [("stream", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_size_t), ("architecture", ctypes.c_int32),
                ("kernel_family", ctypes.c_int32), ("implementation_id", ctypes.c_uint32)]


class RRRouteTraceInfo(ctypes.Structure):
    _fields_ = [("tokens", ctypes.c_int32), ("experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("frame_count", ctypes.c_int32),
                ("trace_id", ctypes.c_char * 128), ("source_kind", ctypes.c_char * 32),
                ("frame_id", ctypes.c_char * 128)]


@dataclasses.dataclass
class Context:
    """Mirror of raggedroute::RuntimeContext plus the KernelSelection."""
    stream: int = 0            # cudaStream_t as an integer (torch.cuda.Stream.cuda_stream)
    workspace: int = 0         # device pointer
    workspace_bytes: int = 0
    architecture: int = ARCH_AUTO
    kernel_family: int = FAMILY_AUTO
    implementation_id: int = 0

    def as_c(self) -> RRContext:
        return RRContext(self.stream or None, self.workspace or None, self.workspace_bytes,
                         self.architecture, self.kernel_family, self.implementation_id)


_P = ctypes.c_void_p
_I = ctypes.c_int
_CTX = ctypes.POINTER(RRContext)

# name -> (restype, argtypes); every rr_* symbol of include/raggedroute_b200.h.
SIGNATURES = {
    "rr_dense_gemm": (RRStatus, [_P, _P, _P, _I, _I, _I, _CTX]),
    "rr_dense_gemm_workspace_size": (ctypes.c_size_t, [_I, _I, _I]),
    "rr_topk_gate": (RRStatus, [_P, _P, _P, _I, _I, _I, _CTX]),
    "rr_topk_gate_workspace_size": (ctypes.c_size_t, [_I, _I]),
    "rr_topk_gate_biased": (RRStatus, [_P, _P, _P, _P, _I, _I, _I, _CTX]),
    "rr_histogram": (RRStatus, [_P, _P, _I, _I, _CTX]),
    "rr_histogram_workspace_size": (ctypes.c_size_t, [_I, _I]),
    "rr_exclusive_scan": (RRStatus, [_P, _P, _I, _CTX]),
    "rr_exclusive_scan_workspace_size": (ctypes.c_size_t, [_I]),
    "rr_histogram_exclusive_scan": (RRStatus, [_P, _P, _P, _I, _I, _CTX]),
    "rr_histogram_exclusive_scan_workspace_size": (ctypes.c_size_t, [_I, _I]),
    "rr_token_permute": (RRStatus, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _CTX]),
    "rr_token_permute_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "rr_token_permute_no_alloc": (RRStatus, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _CTX]),
    "rr_grouped_gemm": (RRStatus, [_P, _P, _P, _P, _I, _I, _I, _I, _CTX]),
    "rr_grouped_gemm_workspace_size": (ctypes.c_size_t, [_I, _I, _I]),
    "rr_unpermute": (RRStatus, [_P, _P, _P, _P, _I, _I, _I, _CTX]),
    "rr_unpermute_workspace_size": (ctypes.c_size_t, [_I, _I, _I]),
    "rr_chain_from_tokens": (RRStatus, [_P] * 13 + [_I] * 4 + [_CTX]),
    "rr_grouped_gemm_gather": (RRStatus, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _CTX]),
    "rr_grouped_gemm_combine": (RRStatus, [_P] * 6 + [_I] * 6 + [_CTX]),
    "rr_grouped_gemm_scatter": (RRStatus, [_P] * 5 + [_I, ctypes.c_int64] + [_I] * 4 + [_CTX]),
    "rr_prepared_expert_weights_size": (ctypes.c_size_t, [_I, _I, _I]),
    "rr_prepare_expert_weights": (RRStatus, [_P, _I, _I, _I, _P, ctypes.c_size_t, _CTX]),
    "rr_grouped_gemm_prepared": (RRStatus, [_P, _P, _P, _P, _I, _I, _I, _I, _CTX]),
    "rr_chain_from_route_ids": (RRStatus, [_P] * 11 + [_I] * 5 + [_CTX]),
    "rr_route_chain_workspace_size": (ctypes.c_size_t, [_I, _I, _I]),
    "rr_chain_from_logits": (RRStatus, [_P] * 11 + [_I] * 4 + [_CTX]),
    "rr_chain_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "rr_launch_dense_gemm_naive": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "rr_launch_topk_gate_naive": (_I, [_P, _P, _P, _I, _I, _P]),
    "rr_launch_histogram_naive": (_I, [_P, _P, _I, _I, _P]),
    "rr_launch_exclusive_scan_naive": (_I, [_P, _P, _I, _P]),
    "rr_launch_token_permute_naive": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "rr_launch_grouped_gemm_naive": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "rr_launch_unpermute_naive": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "rr_launch_cache_scrub": (_I, [_P, ctypes.c_size_t, _P]),
    "rr_classify_compute_capability": (ctypes.c_int32, [_I, _I]),
    "rr_query_current_device_architecture": (RRStatus, [ctypes.POINTER(ctypes.c_int32)]),
    "rr_kernel_launch_count": (ctypes.c_uint64, []),
    "rr_consume_device_error": (RRStatus, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "rr_grouped_gemm_engine": (_I, [_P, _P, _P, _I, _I]),
    "rr_tf32_rounding_selfcheck": (RRStatus, [_P, ctypes.c_int64, _P, _P]),
    "rr_bounded_wait_selftest": (RRStatus, [ctypes.c_uint64, _P, _P]),
    "rr_version": (ctypes.c_char_p, []),
    "rr_route_trace_read": (RRStatus, [ctypes.c_char_p, _I, ctypes.POINTER(RRRouteTraceInfo),
                                          _P, ctypes.c_int64]),
    "rr_route_trace_logits": (RRStatus, [_P, _I, _I, _P]),
    "rr_graph_capture_begin": (RRStatus, [_P]),
    "rr_graph_capture_end": (RRStatus, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "rr_graph_launch": (RRStatus, [_P, _P]),
    "rr_graph_node_count": (_I, [_P]),
    "rr_graph_destroy": (RRStatus, [_P]),
    "rr_host_chain_create": (RRStatus, [_I, _I, _I, _I, ctypes.POINTER(ctypes.c_void_p)]),
    "rr_host_chain_destroy": (RRStatus, [_P]),
    "rr_host_chain_set_flags": (RRStatus, [_P, ctypes.c_uint32]),
    "rr_chain_from_tokens_host": (RRStatus, [_P] * 8 + [_I, _CTX]),
    "rr_ep_get_unique_id": (RRStatus, [_P]),
    "rr_ep_create": (RRStatus, [_P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_double, _I,
                                 ctypes.POINTER(ctypes.c_void_p)]),
    "rr_ep_transport": (RRStatus, [_P, ctypes.POINTER(ctypes.c_int)]),
    "rr_ep_destroy": (RRStatus, [_P]),
    "rr_ep_chain_from_tokens": (RRStatus, [_P] * 15 + [_I, _CTX]),
    "rr_ep_last_step_rows": (RRStatus, [_P, ctypes.POINTER(ctypes.c_int64),
                                        ctypes.POINTER(ctypes.c_int64)]),
    "rr_ep_plan": (RRStatus, [_P, _I, _I, _I, _P, _P, _P, _P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libraggedroute_b200.so (raises if it is missing or unloadable)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(library_path):
                raise RaggedRouteError(int(StatusCode.CUDA_ERROR), 0,
                                       f"{library_path} is missing; run "
                                       "`python -m raggedroute_b200.build`", "load")
            handle = ctypes.CDLL(library_path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def check(status: RRStatus, op: str) -> None:
    if status.code != 0:
        msg = status.message.decode() if status.message else "error"
        raise RaggedRouteError(status.code, status.cuda_error, msg, op)
