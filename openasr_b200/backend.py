"""Python host mirror of the backend operator interface.

Mirrors the calls openasr-core's ggml runtime makes for the hot path
(crates/openasr-core/src/ggml_runtime/cpu_graph.rs: mul_mat :3616,
mul_mat_with_precision :3624, flash_attn_ext :4122,
flash_attn_ext_with_precision :4144, set_rows :4882, top1_argmax_first_max
:3752) and its status mapping (:8380-8405), over the C ABI in
include/oasr_b200.h.  Device memory and streams come from PyTorch tensors; all
arithmetic runs in liboasr_b200.so.  There is no CPU fallback: importing this
module fails if the library is missing.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboasr_b200.so")

F32, F16, Q4_0, Q8_0, Q4_K, I32, I64 = 0, 1, 2, 8, 12, 26, 27
PREC_DEFAULT, PREC_F32 = 0, 10
OP_MUL_MAT, OP_FLASH_ATTN_EXT, OP_SET_ROWS, OP_ARGMAX_FIRST = 1, 2, 3, 4

STATUS_ALLOC_FAILED, STATUS_FAILED, STATUS_SUCCESS = -2, -1, 0
STATUS_ABORTED, STATUS_EXECUTION_FAILED, STATUS_DEVICE_LOST, STATUS_BACKEND_POISONED = 1, 2, 3, 4


class GgmlBackendError(RuntimeError):
    """Typed failure of a backend call (cpu_graph.rs:8380-8405 GgmlCpuGraphError)."""

    def __init__(self, status: int, reason: str):
        super().__init__(f"{self.__class__.__name__}(status={status}): {reason}")
        self.status = status
        self.reason = reason


class UnsupportedInputs(GgmlBackendError):
    pass


class AllocFailed(GgmlBackendError):
    pass


class Aborted(GgmlBackendError):
    pass


class ExecutionFailed(GgmlBackendError):
    pass


class DeviceLost(GgmlBackendError):
    pass


class BackendPoisoned(GgmlBackendError):
    pass


_ERRORS = {
    STATUS_FAILED: UnsupportedInputs,
    STATUS_ALLOC_FAILED: AllocFailed,
    STATUS_ABORTED: Aborted,
    STATUS_EXECUTION_FAILED: ExecutionFailed,
    STATUS_DEVICE_LOST: DeviceLost,
    STATUS_BACKEND_POISONED: BackendPoisoned,
}


class OasrTensor(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("data", ctypes.c_void_p),
        ("ne", ctypes.c_int64 * 4),
        ("nb", ctypes.c_int64 * 4),
    ]


class OasrDeviceProps(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 64),
        ("description", ctypes.c_char * 256),
        ("ordinal", ctypes.c_int32),
        ("device_type", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("cc_major", ctypes.c_int32),
        ("cc_minor", ctypes.c_int32),
        ("cancel_mechanism", ctypes.c_int32),
        ("cancel_observation", ctypes.c_int32),
        ("memory_total", ctypes.c_uint64),
        ("memory_free", ctypes.c_uint64),
    ]


class OasrMemStats(ctypes.Structure):
    _fields_ = [
        ("weight_bytes", ctypes.c_uint64),
        ("scratch_bytes", ctypes.c_uint64),
        ("device_total", ctypes.c_uint64),
        ("device_free", ctypes.c_uint64),
        ("n_weights", ctypes.c_int64),
    ]


class OasrNamedTensor(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("type", ctypes.c_int32),
        ("_pad", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("data", ctypes.c_void_p),
        ("bytes", ctypes.c_uint64),
    ]


class OasrWhisperConfig(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int32) for f in
                ("n_mels", "d_model", "n_heads", "n_enc_layers", "n_dec_layers", "n_vocab", "n_audio_ctx",
                 "n_text_ctx", "max_batch")]


class OasrQwenConfig(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int32) for f in
                ("d_model", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "n_vocab", "max_pos",
                 "max_prefill", "max_batch")] + [("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float)]


# ggml_abort_callback: extern "C" fn(*mut c_void) -> bool (ffi.rs:334-336)
ABORT_CB = ctypes.CFUNCTYPE(ctypes.c_bool, ctypes.c_void_p)

# GGML_BACKEND_GRAPH_CANCEL_* (ffi.rs:118-124)
CANCEL_DISABLED, CANCEL_NATIVE, CANCEL_SEGMENTED = 0, 1, 2
CANCEL_OBSERVATION_NONE, CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT, CANCEL_OBSERVATION_GRAPH_COMPLETION = 0, 1, 2


class ServeStats(ctypes.Structure):
    """struct oasr_serve_stats"""
    _fields_ = [(f, ctypes.c_int32) for f in ("steps", "admissions", "width_changes", "max_width")]


class CancelCapability(ctypes.Structure):
    """struct ggml_backend_graph_cancel_capability (ffi.rs:125-131)"""
    _fields_ = [("mechanism", ctypes.c_int32), ("observation_granularity", ctypes.c_int32)]


def valid_cancel_capability(status: int, cap: CancelCapability) -> bool:
    """the pairs the reference host accepts with a terminal status
    (validate_graph_cancel_capability, cpu_graph.rs:7974-8002)"""
    m, o = cap.mechanism, cap.observation_granularity
    pair = ((m, o) == (CANCEL_DISABLED, CANCEL_OBSERVATION_NONE)
            or (m in (CANCEL_SEGMENTED, CANCEL_NATIVE)
                and o in (CANCEL_OBSERVATION_SUBMISSION_CHECKPOINT, CANCEL_OBSERVATION_GRAPH_COMPLETION)))
    return pair and not (status == 0 and m == CANCEL_DISABLED)


# ---- memory API v1 (ffi.rs:144-333; fixed widths of backend_memory.rs:697-704) ----------
MEMORY_ABI_V1 = 1
DOMAIN_DEVICE_LOCAL, DOMAIN_HOST_PAGEABLE, DOMAIN_HOST_PINNED, DOMAIN_UNIFIED, DOMAIN_FILE_BACKED = 1, 2, 3, 4, 5
REQUEST_BUFFER, REQUEST_HOST_IMPORT, REQUEST_GRAPH_PRIVATE, REQUEST_TRANSFER = 1, 2, 3, 4
STATS_BUDGET_UNAVAILABLE = 1
CLAIM_EXACT, CLAIM_CONSERVATIVE_UPPER = 1, 2
MEMORY_HEALTHY, MEMORY_DEGRADED, MEMORY_QUARANTINED, MEMORY_DEVICE_LOST = 0, 1, 2, 3


class MemDomainId(ctypes.Structure):
    _fields_ = [("physical_device_uuid", ctypes.c_uint8 * 16), ("heap_index", ctypes.c_uint32),
                ("kind", ctypes.c_uint32)]


class MemDomain(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("id", MemDomainId),
                ("name", ctypes.c_char * 48)]


class MemRequest(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("kind", ctypes.c_uint32), ("flags", ctypes.c_uint32),
                ("usage", ctypes.c_uint32), ("request_id", ctypes.c_uint64), ("backend", ctypes.c_void_p),
                ("peer_backend", ctypes.c_void_p), ("buft", ctypes.c_void_p), ("graph", ctypes.c_void_p),
                ("host_ptr", ctypes.c_void_p), ("requested_bytes", ctypes.c_uint64),
                ("currently_allocated_bytes", ctypes.c_uint64), ("max_tensor_bytes", ctypes.c_uint64)]


class MemClaim(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("request_id", ctypes.c_uint64),
                ("domain", MemDomainId)] + [(f, ctypes.c_uint64) for f in (
                    "payload_requested_bytes", "committed_before_bytes", "committed_after_upper_bytes",
                    "commit_peak_extra_upper_bytes", "resident_after_upper_bytes", "retained_after_use_upper_bytes",
                    "releasable_after_use_upper_bytes")]


class MemQuote(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("residual_flags", ctypes.c_uint32),
                ("residual_request_count", ctypes.c_uint32), ("provisional_requested_upper_bytes", ctypes.c_uint64),
                ("stats_generation", ctypes.c_uint64), ("quote_token", ctypes.c_uint64),
                ("request_fingerprint", ctypes.c_uint64)]


class MemStats(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("domain", MemDomainId)] + [
        (f, ctypes.c_uint64) for f in (
            "generation", "timestamp_monotonic_ns", "total_bytes", "budget_bytes", "device_used_bytes",
            "device_free_bytes", "backend_owned_live_bytes", "backend_owned_cached_bytes",
            "backend_owned_workspace_bytes", "backend_owned_high_water_bytes", "allocation_count",
            "allocation_failure_count")] + [
        ("health", ctypes.c_uint32), ("last_ggml_status", ctypes.c_int32), ("last_native_error", ctypes.c_int64),
        ("quarantine_generation", ctypes.c_uint64)]


class MemQuarantine(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("reason", ctypes.c_uint32),
                ("ggml_status", ctypes.c_int32), ("native_error", ctypes.c_int64), ("message", ctypes.c_char * 96)]


_U32P = ctypes.POINTER(ctypes.c_uint32)
MEM_GET_DOMAINS = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(MemDomain), _U32P)
MEM_QUOTE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(MemRequest), ctypes.c_uint32, ctypes.POINTER(MemQuote),
                             ctypes.POINTER(MemClaim), _U32P)
MEM_RESERVE_PRIVATE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(MemRequest), ctypes.c_uint32,
                                       ctypes.POINTER(MemQuote), ctypes.POINTER(MemClaim), _U32P)
MEM_GET_STATS = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(MemStats), _U32P)
MEM_TRIM = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64)
MEM_QUARANTINE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(MemQuarantine))


class MemoryApiV1(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32), ("capabilities", ctypes.c_uint64),
                ("get_domains", MEM_GET_DOMAINS), ("quote", MEM_QUOTE), ("reserve_private", MEM_RESERVE_PRIVATE),
                ("get_stats", MEM_GET_STATS), ("trim", MEM_TRIM), ("quarantine", MEM_QUARANTINE)]


def memory_api() -> MemoryApiV1:
    """The table ggml_backend_memory_get_api_v1 returns (static for the process)."""
    return lib().oasr_b200_memory_get_api_v1().contents


def _counted(call, item_type):
    """The v1 count protocol: size with a null array, then fill (backend_memory.rs:193-356)."""
    n = ctypes.c_uint32(0)
    rc = call(None, ctypes.byref(n))
    if rc != 0:
        return rc, []
    items = (item_type * max(n.value, 1))()
    for it in items:
        it.struct_size = ctypes.sizeof(item_type)
    cap = ctypes.c_uint32(n.value)
    rc = call(items, ctypes.byref(cap))
    return rc, list(items)[: cap.value] if rc == 0 else []

# every symbol include/oasr_b200.h declares, with (argtypes, restype)
_P, _I32, _I64, _U64, _F, _SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_size_t
_TP = ctypes.POINTER(OasrTensor)
SIGNATURES = {
    "oasr_b200_device_count": ([ctypes.POINTER(_I32)], ctypes.c_int),
    "oasr_b200_init": ([_I32, ctypes.POINTER(_P)], ctypes.c_int),
    "oasr_b200_free": ([_P], ctypes.c_int),
    "oasr_b200_props": ([_P, ctypes.POINTER(OasrDeviceProps)], ctypes.c_int),
    "oasr_b200_supports_op": ([_P, _I32, _TP, _TP], ctypes.c_int),
    "oasr_b200_set_stream": ([_P, _P], ctypes.c_int),
    "oasr_b200_get_stream": ([_P], _P),
    "oasr_b200_synchronize": ([_P], ctypes.c_int),
    "oasr_b200_synchronize_ex": ([_P, ctypes.POINTER(CancelCapability)], ctypes.c_int),
    "oasr_b200_get_proc_address": ([ctypes.c_char_p], _P),
    "oasr_b200_selftest_bounded_wait": ([_P, _I64], ctypes.c_int),
    "oasr_b200_set_abort_callback": ([_P, ABORT_CB, _P], ctypes.c_int),
    "oasr_b200_mem_stats": ([_P, ctypes.POINTER(OasrMemStats)], ctypes.c_int),
    "oasr_b200_last_error": ([_P], ctypes.c_char_p),
    "oasr_b200_reserve_scratch": ([_P, _SZ], ctypes.c_int),
    "oasr_b200_weight_upload": ([_P, _P, _SZ, _I32, ctypes.POINTER(_I64), ctypes.POINTER(_P)], ctypes.c_int),
    "oasr_b200_weight_free": ([_P, _P], ctypes.c_int),
    "oasr_b200_weight_download": ([_P, _P, _P, _SZ], ctypes.c_int),
    "oasr_b200_weight_info": ([_P, ctypes.POINTER(_I32), ctypes.POINTER(_I64), ctypes.POINTER(_U64)], ctypes.c_int),
    "oasr_b200_mul_mat": ([_P, _P, _TP, _TP, _I32], ctypes.c_int),
    "oasr_b200_act_bytes": ([_I32, _I64, _I64], _I64),
    "oasr_b200_quantize_act": ([_P, _I32, _TP, _P, _SZ], ctypes.c_int),
    "oasr_b200_mul_mat_qact": ([_P, _P, _P, _I64, _TP], ctypes.c_int),
    "oasr_b200_flash_attn_ext": ([_P, _TP, _TP, _TP, _TP, _F, _F, _F, _I32, _TP], ctypes.c_int),
    "oasr_b200_flash_attn_ext_static": ([_P, _TP, _TP, _TP, _TP, _F, _F, _F, _I32, _TP], ctypes.c_int),
    "oasr_b200_flash_attn_causal": ([_P, _TP, _TP, _TP, _F, _I32, _TP], ctypes.c_int),
    "oasr_b200_set_rows": ([_P, _TP, _TP, _TP], ctypes.c_int),
    "oasr_b200_argmax_first": ([_P, _TP, _TP], ctypes.c_int),
    "oasr_b200_whisper_load": ([_P, ctypes.POINTER(OasrWhisperConfig), ctypes.POINTER(OasrNamedTensor), _I32,
                                ctypes.POINTER(_P)], ctypes.c_int),
    "oasr_b200_whisper_free": ([_P], ctypes.c_int),
    "oasr_b200_whisper_mel": ([_P, _P, _P, _I32, _P], ctypes.c_int),
    "oasr_b200_whisper_encode": ([_P, _P, _I32, _P], ctypes.c_int),
    "oasr_b200_whisper_decode_step": ([_P, _P, _I32, _I32, _P, _P], ctypes.c_int),
    "oasr_b200_whisper_transcribe": ([_P, _P, _P, _I32, _P, _I32, _I32, _I32, _I32, _P], ctypes.c_int),
    "oasr_b200_whisper_mel_device": ([_P, _P, _P, _I32], ctypes.c_int),
    "oasr_b200_whisper_max_batch": ([_P], ctypes.c_int32),
    "oasr_b200_whisper_serve": ([_P, _P, _P, _I32, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _P, _P,
                                 ctypes.POINTER(ServeStats)], ctypes.c_int),
    "oasr_b200_serve_batch_width": ([_I32, _I32], ctypes.c_int32),
    "oasr_b200_serve_batch_vram_cap": ([_I32, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int32),
    "oasr_b200_whisper_generate": ([_P, _I32, _P, _I32, _I32, _I32, _I32, _P, _I32], ctypes.c_int),
    "oasr_b200_qwen_load": ([_P, ctypes.POINTER(OasrQwenConfig), ctypes.POINTER(OasrNamedTensor), _I32,
                             ctypes.POINTER(_P)], ctypes.c_int),
    "oasr_b200_qwen_free": ([_P], ctypes.c_int),
    "oasr_b200_qwen_prefill": ([_P, _P, _I32, _I32, _I32, _P, _P], ctypes.c_int),
    "oasr_b200_qwen_decode_step": ([_P, _P, _I32, _I32, _P, _P], ctypes.c_int),
    "oasr_b200_qwen_generate": ([_P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I32], ctypes.c_int),
    "oasr_b200_qwen_read_kv": ([_P, _I32, _I32, _I32, _P, _P], ctypes.c_int),
    "oasr_b200_row_size": ([_I32, _I64], _I64),
    "oasr_b200_quantize_chunk": ([_I32, _P, _P, _I64, _I64, _I64], _I64),
    "oasr_b200_synth_normal": ([_U64, _U64, _P, _I64, _F, _F], ctypes.c_int),
    "oasr_b200_memory_get_api_v1": ([], ctypes.POINTER(MemoryApiV1)),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load liboasr_b200.so (raises if it has not been built: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m openasr_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes, fn.restype = args, res
        _lib = L
    return _lib


# ---- host helpers (no device) -----------------------------------------------------------
def row_size(ggml_type: int, ne0: int) -> int:
    return int(lib().oasr_b200_row_size(ggml_type, ne0))


def quantize(ggml_type: int, x: np.ndarray) -> np.ndarray:
    """ggml_quantize_chunk over the rows of a 2-D f32 array -> uint8 (rows, row_bytes)."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    rows, n = x.shape
    rs = row_size(ggml_type, n)
    if rs < 0:
        raise UnsupportedInputs(STATUS_FAILED, f"row of {n} elements is not a multiple of the block size")
    out = np.empty((rows, rs), np.uint8)
    got = lib().oasr_b200_quantize_chunk(ggml_type, x.ctypes.data, out.ctypes.data, 0, rows, n)
    if got != rows * rs:
        raise UnsupportedInputs(STATUS_FAILED, f"quantize_chunk returned {got}")
    return out


def synth_normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    rc = lib().oasr_b200_synth_normal(seed & (2**64 - 1), offset, out.ctypes.data, n, mean, std)
    if rc != 0:
        raise UnsupportedInputs(rc, "synth_normal")
    return out


# ---- tensor descriptors -----------------------------------------------------------------
_TORCH_TYPES = None


def _torch_type(t) -> int:
    import torch

    m = {torch.float32: F32, torch.float16: F16, torch.int32: I32, torch.int64: I64}
    if t.dtype not in m:
        raise UnsupportedInputs(STATUS_FAILED, f"unsupported tensor dtype {t.dtype}")
    return m[t.dtype]


def describe(t, ggml_type: int | None = None) -> OasrTensor:
    """oasr_tensor for a torch tensor: ne = reversed shape, nb = reversed byte strides."""
    d = OasrTensor()
    d.type = _torch_type(t) if ggml_type is None else ggml_type
    d.flags = 0
    d.data = t.data_ptr()
    shape = list(t.shape)[::-1] + [1] * (4 - t.dim())
    es = t.element_size()
    strides = [s * es for s in list(t.stride())[::-1]]
    while len(strides) < 4:
        strides.append(strides[-1] * shape[len(strides) - 1] if strides else es)
    d.ne[:] = shape[:4]
    d.nb[:] = strides[:4]
    return d


class Weight:
    """A resident quantized weight (ggml [K, N, ne2, ne3])."""

    def __init__(self, backend: "Backend", handle: int, ggml_type: int, ne):
        self.backend = backend
        self.handle = ctypes.c_void_p(handle)
        self.type = ggml_type
        self.ne = list(ne)

    @property
    def K(self) -> int:
        return self.ne[0]

    @property
    def N(self) -> int:
        return self.ne[1]

    def device_bytes(self) -> int:
        nb = ctypes.c_uint64()
        lib().oasr_b200_weight_info(self.handle, None, None, ctypes.byref(nb))
        return nb.value

    def download(self) -> np.ndarray:
        rows = self.ne[1] * self.ne[2] * self.ne[3]
        out = np.empty((rows, row_size(self.type, self.ne[0])), np.uint8)
        self.backend._check(lib().oasr_b200_weight_download(self.backend.handle, self.handle, out.ctypes.data, out.nbytes))
        return out

    def free(self) -> None:
        if self.handle:
            lib().oasr_b200_weight_free(self.backend.handle, self.handle)
            self.handle = ctypes.c_void_p(0)


class Backend:
    """One device + one stream (ggml_backend_dev_init / ggml_backend_t)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        rc = lib().oasr_b200_init(ordinal, ctypes.byref(h))
        if rc != 0:
            raise _ERRORS.get(rc, GgmlBackendError)(rc, f"oasr_b200_init({ordinal}) failed")
        self.handle = h
        self.ordinal = ordinal
        self._abort_cb = None
        self.own_stream = lib().oasr_b200_get_stream(h) or 0

    # -- status mapping (cpu_graph.rs:8380-8405) --
    def _check(self, rc: int) -> None:
        if rc != 0:
            reason = lib().oasr_b200_last_error(self.handle)
            raise _ERRORS.get(rc, GgmlBackendError)(rc, reason.decode() if reason else "")

    def close(self) -> None:
        if self.handle:
            lib().oasr_b200_free(self.handle)
            self.handle = ctypes.c_void_p(0)

    def props(self) -> dict:
        p = OasrDeviceProps()
        self._check(lib().oasr_b200_props(self.handle, ctypes.byref(p)))
        return {f: (getattr(p, f).decode() if isinstance(getattr(p, f), bytes) else getattr(p, f)) for f, _ in p._fields_}

    def mem_stats(self) -> dict:
        s = OasrMemStats()
        self._check(lib().oasr_b200_mem_stats(self.handle, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in s._fields_}

    def set_stream(self, stream) -> None:
        """Enqueue on a torch.cuda.Stream or a raw cudaStream_t (int; 0 is the
        legacy default stream); None returns to the backend's own stream."""
        if stream is None:
            ptr = self.own_stream
        else:
            ptr = stream if isinstance(stream, int) else stream.cuda_stream
        self._check(lib().oasr_b200_set_stream(self.handle, ptr))

    def stream_ptr(self) -> int:
        return lib().oasr_b200_get_stream(self.handle) or 0

    def synchronize(self) -> None:
        self._check(lib().oasr_b200_synchronize(self.handle))

    def synchronize_ex(self) -> tuple[int, CancelCapability]:
        """(merged status, cancel capability) as ggml_backend_graph_compute_with_abort
        reports them; the status is returned, not raised"""
        cap = CancelCapability()
        rc = lib().oasr_b200_synchronize_ex(self.handle, ctypes.byref(cap))
        return rc, cap

    # -- memory API v1 (the table a plugin loader resolves by proc address) --
    def memory_domains(self) -> list:
        api = memory_api()
        rc, items = _counted(lambda arr, n: api.get_domains(self.handle, arr, n), MemDomain)
        self._check(rc)
        return items

    def memory_stats(self) -> list:
        api = memory_api()
        rc, items = _counted(lambda arr, n: api.get_stats(self.handle, self.handle, arr, n), MemStats)
        self._check(rc)
        return items

    def memory_request(self, kind: int, nbytes: int, request_id: int = 0, usage: int = 0) -> MemRequest:
        r = MemRequest()
        r.struct_size = ctypes.sizeof(MemRequest)
        r.kind, r.usage, r.request_id, r.requested_bytes = kind, usage, request_id, nbytes
        r.backend = self.handle
        return r

    def memory_quote(self, requests) -> tuple:
        """(quote, claims) for a list of MemRequest."""
        api = memory_api()
        arr = (MemRequest * max(len(requests), 1))(*requests)
        q = MemQuote()
        q.struct_size = ctypes.sizeof(MemQuote)
        rc, claims = _counted(lambda c, n: api.quote(arr, len(requests), ctypes.byref(q), c, n), MemClaim)
        self._check(rc)
        return q, claims

    def memory_reserve_private(self, requests, quote: MemQuote, sizing_only: bool = False):
        """Commit the backend-private requests of `quote`; returns the actual claims (or,
        with sizing_only, just their count)."""
        api = memory_api()
        arr = (MemRequest * max(len(requests), 1))(*requests)
        n = ctypes.c_uint32(0)
        self._check(api.reserve_private(arr, len(requests), ctypes.byref(quote), None, ctypes.byref(n)))
        if sizing_only:
            return n.value
        claims = (MemClaim * max(n.value, 1))()
        for c in claims:
            c.struct_size = ctypes.sizeof(MemClaim)
        cap = ctypes.c_uint32(n.value)
        self._check(api.reserve_private(arr, len(requests), ctypes.byref(quote), claims, ctypes.byref(cap)))
        return list(claims)[: cap.value]

    def memory_trim(self, flags: int = 0) -> None:
        self._check(memory_api().trim(self.handle, flags))

    def memory_quarantine(self, status: int, message: str, native_error: int = 0) -> None:
        q = MemQuarantine()
        q.struct_size = ctypes.sizeof(MemQuarantine)
        q.ggml_status, q.native_error = status, native_error
        q.message = message.encode()[:95]
        self._check(memory_api().quarantine(self.handle, ctypes.byref(q)))

    def reserve_scratch(self, nbytes: int) -> None:
        self._check(lib().oasr_b200_reserve_scratch(self.handle, nbytes))

    def set_abort_callback(self, fn) -> None:
        """fn() -> bool; polled before every enqueue (ggml_abort_callback)."""
        if fn is None:
            self._abort_cb = None
            self._check(lib().oasr_b200_set_abort_callback(self.handle, ABORT_CB(0), None))
            return
        self._abort_cb = ABORT_CB(lambda _data: bool(fn()))
        self._check(lib().oasr_b200_set_abort_callback(self.handle, self._abort_cb, None))

    def supports_op(self, op: int, src0: OasrTensor, src1: OasrTensor | None = None) -> bool:
        return bool(lib().oasr_b200_supports_op(self.handle, op, ctypes.byref(src0),
                                                ctypes.byref(src1) if src1 is not None else None))

    def device_supports_matmul_for_type(self, ggml_type: int) -> bool:
        """backend.rs:295-323: probe mul_mat(W[K=256, N=32] of type T, X f32 [256, 8])."""
        w = OasrTensor(type=ggml_type, data=None)
        w.ne[:] = [256, 32, 1, 1]
        x = OasrTensor(type=F32, data=None)
        x.ne[:] = [256, 8, 1, 1]
        return self.supports_op(OP_MUL_MAT, w, x)

    # -- weights (cpu_graph.rs:9497 maybe_allocate_weight_buffer_from_host_ptr) --
    def upload_weight(self, blocks: np.ndarray, ggml_type: int, ne) -> Weight:
        blocks = np.ascontiguousarray(blocks)
        ne = list(ne) + [1] * (4 - len(ne))
        arr = (ctypes.c_int64 * 4)(*ne)
        h = ctypes.c_void_p()
        self._check(lib().oasr_b200_weight_upload(self.handle, blocks.ctypes.data, blocks.nbytes, ggml_type, arr,
                                                  ctypes.byref(h)))
        return Weight(self, h.value, ggml_type, ne)

    # -- ops --
    def mul_mat(self, w: Weight, x, out, prec: int = PREC_DEFAULT) -> None:
        self._check(lib().oasr_b200_mul_mat(self.handle, w.handle, ctypes.byref(describe(x)), ctypes.byref(describe(out)), prec))

    @staticmethod
    def act_bytes(weight_type: int, K: int, rows: int) -> int:
        n = int(lib().oasr_b200_act_bytes(weight_type, K, rows))
        if n < 0:
            raise UnsupportedInputs(n, "act_bytes: unsupported weight type or K")
        return n

    def quantize_act(self, weight_type: int, x, qact) -> None:
        """Convert x (f32|f16 [rows, K]) into qact (a uint8 CUDA tensor of act_bytes)."""
        self._check(lib().oasr_b200_quantize_act(self.handle, weight_type, ctypes.byref(describe(x)), qact.data_ptr(),
                                                 qact.numel() * qact.element_size()))

    def mul_mat_qact(self, w: Weight, qact, rows: int, out) -> None:
        self._check(lib().oasr_b200_mul_mat_qact(self.handle, w.handle, qact.data_ptr(), rows, ctypes.byref(describe(out))))

    def flash_attn_ext(self, q, k, v, mask, scale: float, out, max_bias: float = 0.0, logit_softcap: float = 0.0,
                       prec: int = PREC_DEFAULT) -> None:
        md = describe(mask) if mask is not None else None
        self._check(lib().oasr_b200_flash_attn_ext(
            self.handle, ctypes.byref(describe(q)), ctypes.byref(describe(k)), ctypes.byref(describe(v)),
            ctypes.byref(md) if md is not None else None, scale, max_bias, logit_softcap, prec, ctypes.byref(describe(out))))

    def flash_attn_ext_static(self, q, k, v, mask, scale: float, out, max_bias: float = 0.0,
                              logit_softcap: float = 0.0, prec: int = PREC_DEFAULT) -> None:
        """flash_attn_ext over file-scope device scratch: allocates nothing; overlapping
        calls on one device race (see the C header)."""
        md = describe(mask) if mask is not None else None
        self._check(lib().oasr_b200_flash_attn_ext_static(
            self.handle, ctypes.byref(describe(q)), ctypes.byref(describe(k)), ctypes.byref(describe(v)),
            ctypes.byref(md) if md is not None else None, scale, max_bias, logit_softcap, prec, ctypes.byref(describe(out))))

    def flash_attn_causal(self, q, k, v, scale: float, out, prec: int = PREC_DEFAULT) -> None:
        """flash_attn_ext under the causal mask (key j visible to query i when
        j <= i + n_kv - n_q) on the tensor cores; no mask tensor."""
        self._check(lib().oasr_b200_flash_attn_causal(
            self.handle, ctypes.byref(describe(q)), ctypes.byref(describe(k)), ctypes.byref(describe(v)), scale, prec,
            ctypes.byref(describe(out))))

    def set_rows(self, dst, src, rows) -> None:
        self._check(lib().oasr_b200_set_rows(self.handle, ctypes.byref(describe(dst)), ctypes.byref(describe(src)),
                                             ctypes.byref(describe(rows))))

    def argmax_first(self, logits, out) -> None:
        self._check(lib().oasr_b200_argmax_first(self.handle, ctypes.byref(describe(logits)), ctypes.byref(describe(out))))


def device_count() -> int:
    n = ctypes.c_int32()
    lib().oasr_b200_device_count(ctypes.byref(n))
    return n.value
