"""Python host mirror of the julia1-rs engine API over libj1 (ctypes).

The reference's Rust API (crate `julia1`, src/lib.rs) exposes `Engine`,
`EngineOptions`, `Device` and, below the tokenizer, `Engine::logits_encoded`
over `encode::Encoded` rows. This module mirrors those names on top of the C ABI
in include/j1.h; all compute runs in libj1's CUDA kernels. There is no CPU
fallback: if lib/libj1.so is missing or the device is not an sm_100 GPU, calls
raise J1Error.
"""
import ctypes as C
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libj1.so")

OK, INVALID_ARG, UNSUPPORTED, CUDA, OOM, NONFINITE, DEVICE_TIMEOUT, IO, INTERNAL = range(9)
STATUS_NAMES = ["J1_OK", "J1_ERR_INVALID_ARG", "J1_ERR_UNSUPPORTED", "J1_ERR_CUDA", "J1_ERR_OOM",
                "J1_ERR_NONFINITE", "J1_ERR_DEVICE_TIMEOUT", "J1_ERR_IO", "J1_ERR_INTERNAL"]

# Every symbol include/j1.h declares (checked by tests against the built library).
EXPORTS = [
    "j1_last_error", "j1_status_name", "j1_version", "j1_config_load",
    "j1_model_create", "j1_model_destroy", "j1_model_name", "j1_model_config", "j1_model_forward",
    "j1_model_stage", "j1_model_launch", "j1_model_finish", "j1_model_stream", "j1_model_launch_count",
    "j1_model_forward_many",
    "j1_engine_options_default", "j1_engine_create", "j1_engine_create_pool", "j1_engine_destroy",
    "j1_engine_device_name", "j1_engine_logits_encoded",
    "j1_op_gemm", "j1_op_attention", "j1_op_attention_noalloc", "j1_op_geglu_interleave",
    "j1_model_profile", "j1_model_profile_read", "j1_profile_family_name", "j1_plan_batches",
    "j1_engine_max_length", "j1_encoder_options_default", "j1_encode_sequence", "j1_engine_logits_tokenized",
    "j1_router_options_default", "j1_router_create", "j1_router_create_with_scorer", "j1_router_destroy",
    "j1_router_clear_cache", "j1_router_route_many", "j1_display_probabilities", "j1_router_confident_winner",
    "j1_tokenizer_load", "j1_tokenizer_from_json", "j1_tokenizer_destroy", "j1_tokenizer_token_to_id",
    "j1_tokenizer_encode", "j1_tokenizer_encode_batch", "j1_text_encoder_load", "j1_text_encoder_destroy",
    "j1_text_encoder_clear_cache", "j1_text_encoder_options", "j1_text_encoder_tokenize", "j1_text_encoder_encode",
    "j1_text_encoder_request_tokens", "j1_text_encoder_encode_batch", "j1_engine_logits_text", "j1_json_dumps",
    "j1_inject_fault", "j1_selftest_device_timeout",
]
FAULT_ALLOC, FAULT_LAUNCH, FAULT_NAN, FAULT_HOST, FAULT_WORKER, FAULT_THREAD, FAULT_DEVICE_WAIT = 1, 2, 3, 4, 5, 6, 7
PROF_FAMILIES = 12

EPI_BF16, EPI_QKV_ROPE, EPI_GEGLU, EPI_RESID_LN, EPI_RESID, EPI_SCORER = range(6)


class J1Error(RuntimeError):
    def __init__(self, status, message):
        self.status = status
        super().__init__("%s: %s" % (STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else status, message))


class J1Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "heads", "head_dim", "intermediate", "layers", "half_window",
                                         "vocab", "max_positions", "head_layers", "head_heads", "head_ff")] + \
               [("norm_eps", C.c_float), ("n_global", C.c_int32)]


class J1Batch(C.Structure):
    _fields_ = [("ids", C.POINTER(C.c_uint32)), ("t", C.c_size_t), ("starts", C.POINTER(C.c_uint32)),
                ("lens", C.POINTER(C.c_uint32)), ("qtypes", C.POINTER(C.c_uint8)), ("nseq", C.c_size_t),
                ("marker_rows", C.POINTER(C.c_uint32)), ("marker_starts", C.POINTER(C.c_uint32)), ("m", C.c_size_t)]


class J1EngineOptions(C.Structure):
    _fields_ = [("device", C.c_char_p), ("batch_size", C.c_int32), ("max_batch_tokens", C.c_int64),
                ("max_length", C.c_int32)]


class J1GemmArgs(C.Structure):
    _fields_ = [("epilogue", C.c_int32), ("M", C.c_int32), ("N", C.c_int32), ("K", C.c_int32),
                ("A", C.c_void_p), ("W", C.c_void_p), ("out", C.c_void_p), ("ldo", C.c_int32),
                ("bias", C.c_void_p), ("relu", C.c_int32), ("x", C.c_void_p), ("ldx", C.c_int32),
                ("ln_w", C.c_void_p), ("ln_b", C.c_void_p), ("ln_eps", C.c_float), ("xn", C.c_void_p),
                ("ldxn", C.c_int32), ("pos", C.c_void_p), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
                ("rope_cols", C.c_int32), ("w2", C.c_void_p), ("b2", C.c_float), ("scores", C.c_void_p),
                ("grid_limit", C.c_int32)]


class J1EncoderOptions(C.Structure):
    _fields_ = [("cls_id", C.c_uint32), ("sep_id", C.c_uint32), ("mask_id", C.c_uint32), ("max_length", C.c_int32),
                ("head_length", C.c_int32), ("strict", C.c_int32)]


class J1TokenizedRequest(C.Structure):
    _fields_ = [("head_ids", C.POINTER(C.c_uint32)), ("head_len", C.c_size_t),
                ("option_ids", C.POINTER(C.c_uint32)), ("option_lens", C.POINTER(C.c_uint32)),
                ("n_options", C.c_size_t), ("state_ids", C.POINTER(C.c_uint32)), ("state_len", C.c_size_t),
                ("qtype", C.c_uint8)]


class J1RouterOptions(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("width", "survivors", "batch_size", "cache_size", "max_options")]


class J1RouteResult(C.Structure):
    _fields_ = [("index", C.c_uint32), ("n_candidates", C.c_uint32), ("candidates", C.c_uint32 * 20),
                ("probabilities", C.c_double * 20), ("rounds", C.c_uint32), ("hierarchical", C.c_int32)]


class J1TextRequest(C.Structure):
    _fields_ = [("state", C.c_char_p), ("state_is_json", C.c_int32), ("question", C.c_char_p),
                ("options", C.POINTER(C.c_char_p)), ("n_options", C.c_size_t), ("qtype", C.c_uint8)]


_TEXT_DT = np.dtype({"names": ["state", "state_is_json", "question", "options", "n_options", "qtype"],
                     "formats": [np.uint64, np.int32, np.uint64, np.uint64, np.uint64, np.uint8],
                     "offsets": [J1TextRequest.state.offset, J1TextRequest.state_is_json.offset,
                                 J1TextRequest.question.offset, J1TextRequest.options.offset,
                                 J1TextRequest.n_options.offset, J1TextRequest.qtype.offset],
                     "itemsize": C.sizeof(J1TextRequest)})  # j1_text_request, for whole batches at once


def _cstrings(bs):
    """Byte strings as C strings without one ctypes object each: one NUL-separated buffer
    (kept alive by the returned array) and the address of each string."""
    mem = np.frombuffer(b"\0".join(bs) + b"\0", np.uint8)
    lens = np.fromiter(map(len, bs), np.int64, len(bs))
    starts = np.zeros(len(bs), np.int64)
    if len(bs) > 1:
        np.cumsum(lens[:-1] + 1, out=starts[1:])
    return mem, np.uint64(mem.ctypes.data) + starts.astype(np.uint64), lens


SCORER_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                        C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint8), C.POINTER(C.c_float))

_lib = None


def lib():
    """Load libj1.so once (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise J1Error(CUDA, "libj1.so not built (run python julia1-rs_b200/build.py): %s" % LIB_PATH)
    L = C.CDLL(LIB_PATH)
    u32p, f32p, u8p = C.POINTER(C.c_uint32), C.POINTER(C.c_float), C.POINTER(C.c_uint8)
    L.j1_last_error.argtypes = [C.c_char_p, C.c_size_t]
    L.j1_last_error.restype = C.c_size_t
    L.j1_status_name.restype = C.c_char_p
    L.j1_version.restype = C.c_char_p
    L.j1_config_load.argtypes = [C.c_char_p, C.POINTER(J1Config)]
    L.j1_model_create.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_void_p)]
    L.j1_model_destroy.argtypes = [C.c_void_p]
    L.j1_model_destroy.restype = None
    L.j1_model_name.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    L.j1_model_name.restype = C.c_size_t
    L.j1_model_config.argtypes = [C.c_void_p, C.POINTER(J1Config)]
    batch = [u32p, C.c_size_t, u32p, u32p, u8p, C.c_size_t, u32p, u32p, C.c_size_t]
    L.j1_model_forward.argtypes = [C.c_void_p] + batch + [f32p]
    L.j1_model_stage.argtypes = [C.c_void_p] + batch
    L.j1_model_launch.argtypes = [C.c_void_p]
    L.j1_model_finish.argtypes = [C.c_void_p, f32p, C.c_size_t]
    L.j1_model_forward_many.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(J1Batch), C.POINTER(f32p)]
    L.j1_model_forward_many.restype = C.c_int
    L.j1_model_stream.argtypes = [C.c_void_p]
    L.j1_model_stream.restype = C.c_void_p
    L.j1_model_launch_count.argtypes = [C.c_void_p]
    L.j1_model_launch_count.restype = C.c_int64
    L.j1_engine_options_default.argtypes = [C.POINTER(J1EngineOptions)]
    L.j1_engine_options_default.restype = None
    L.j1_engine_create.argtypes = [C.c_char_p, C.POINTER(J1EngineOptions), C.POINTER(C.c_void_p)]
    L.j1_engine_create_pool.argtypes = [C.c_char_p, C.POINTER(J1EngineOptions), C.POINTER(C.c_int), C.c_int,
                                        C.POINTER(C.c_void_p)]
    L.j1_engine_destroy.argtypes = [C.c_void_p]
    L.j1_engine_destroy.restype = None
    L.j1_engine_device_name.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    L.j1_engine_device_name.restype = C.c_size_t
    L.j1_engine_logits_encoded.argtypes = [C.c_void_p, C.c_size_t, u32p, u32p, u32p, u32p, u8p, f32p]
    L.j1_model_profile.argtypes = [C.c_void_p, C.c_int]
    L.j1_model_profile_read.argtypes = [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_int64)]
    L.j1_profile_family_name.argtypes = [C.c_int]
    L.j1_profile_family_name.restype = C.c_char_p
    L.j1_plan_batches.argtypes = [C.c_size_t, u32p, C.c_int32, C.c_int64, C.c_int32, u32p, u32p,
                                  C.POINTER(C.c_size_t)]
    L.j1_plan_batches.restype = C.c_int
    L.j1_engine_max_length.argtypes = [C.c_void_p]
    L.j1_engine_max_length.restype = C.c_int32
    L.j1_encoder_options_default.argtypes = [C.POINTER(J1EncoderOptions)]
    L.j1_encoder_options_default.restype = None
    L.j1_encode_sequence.argtypes = [C.POINTER(J1EncoderOptions), C.POINTER(J1TokenizedRequest), u32p, C.c_size_t,
                                     C.POINTER(C.c_size_t), u32p, C.POINTER(C.c_int32)]
    L.j1_engine_logits_tokenized.argtypes = [C.c_void_p, C.POINTER(J1EncoderOptions), C.c_size_t,
                                             C.POINTER(J1TokenizedRequest), f32p]
    L.j1_router_options_default.argtypes = [C.POINTER(J1RouterOptions)]
    L.j1_router_options_default.restype = None
    L.j1_router_create.argtypes = [C.c_void_p, C.POINTER(J1EncoderOptions), C.POINTER(J1RouterOptions),
                                   C.POINTER(C.c_void_p)]
    L.j1_router_create_with_scorer.argtypes = [SCORER_FN, C.c_void_p, C.POINTER(J1EncoderOptions),
                                               C.POINTER(J1RouterOptions), C.POINTER(C.c_void_p)]
    L.j1_display_probabilities.argtypes = [C.POINTER(C.c_double), C.c_size_t, C.POINTER(C.c_double)]
    L.j1_display_probabilities.restype = None
    L.j1_router_confident_winner.argtypes = [f32p, C.c_size_t, C.c_size_t]
    L.j1_router_confident_winner.restype = C.c_int32
    L.j1_router_destroy.argtypes = [C.c_void_p]
    L.j1_router_destroy.restype = None
    L.j1_router_clear_cache.argtypes = [C.c_void_p]
    L.j1_router_clear_cache.restype = None
    L.j1_router_route_many.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(J1TokenizedRequest),
                                       C.POINTER(J1RouteResult), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    L.j1_tokenizer_load.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.j1_tokenizer_from_json.argtypes = [C.c_char_p, C.c_size_t, C.POINTER(C.c_void_p)]
    L.j1_tokenizer_destroy.argtypes = [C.c_void_p]
    L.j1_tokenizer_destroy.restype = None
    L.j1_tokenizer_token_to_id.argtypes = [C.c_void_p, C.c_char_p]
    L.j1_tokenizer_token_to_id.restype = C.c_int64
    L.j1_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, u32p, C.c_size_t, C.POINTER(C.c_size_t)]
    L.j1_tokenizer_encode_batch.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_char_p), C.POINTER(C.c_size_t),
                                            C.c_int32, u32p, C.c_size_t, C.POINTER(C.c_size_t)]
    L.j1_text_encoder_load.argtypes = [C.c_char_p, C.c_int32, C.c_int32, C.c_int32, C.c_int64, C.c_int64,
                                       C.POINTER(C.c_void_p)]
    L.j1_text_encoder_destroy.argtypes = [C.c_void_p]
    L.j1_text_encoder_destroy.restype = None
    L.j1_text_encoder_clear_cache.argtypes = [C.c_void_p]
    L.j1_text_encoder_clear_cache.restype = None
    L.j1_text_encoder_options.argtypes = [C.c_void_p, C.POINTER(J1EncoderOptions)]
    L.j1_text_encoder_tokenize.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, u32p, C.c_size_t,
                                           C.POINTER(C.c_size_t)]
    L.j1_text_encoder_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_int32, C.c_char_p, C.POINTER(C.c_char_p),
                                         C.c_size_t, C.c_uint8, u32p, C.c_size_t, C.POINTER(C.c_size_t), u32p,
                                         C.POINTER(C.c_int32)]
    L.j1_text_encoder_request_tokens.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.POINTER(C.c_char_p),
                                                 C.c_size_t, C.c_uint8, u32p, C.c_size_t, C.POINTER(C.c_size_t), u32p]
    L.j1_text_encoder_request_tokens.restype = C.c_int
    L.j1_text_encoder_encode_batch.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(J1TextRequest), C.c_int32, u32p,
                                               C.c_size_t, C.POINTER(C.c_size_t), u32p, C.c_size_t,
                                               C.POINTER(C.c_size_t), C.POINTER(C.c_int32)]
    L.j1_text_encoder_encode_batch.restype = C.c_int
    L.j1_engine_logits_text.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(J1TextRequest), C.c_int32,
                                        f32p]
    L.j1_engine_logits_text.restype = C.c_int
    L.j1_json_dumps.argtypes = [C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]
    L.j1_json_dumps.restype = C.c_int
    L.j1_inject_fault.argtypes = [C.c_int32, C.c_int32]
    L.j1_inject_fault.restype = None
    L.j1_selftest_device_timeout.argtypes = [C.c_int, C.c_int64]
    L.j1_selftest_device_timeout.restype = C.c_int
    L.j1_op_gemm.argtypes = [C.POINTER(J1GemmArgs), C.c_void_p, C.c_int]
    L.j1_op_attention.argtypes = [C.c_void_p, C.c_int64, C.c_int32, u32p, u32p, C.c_size_t, C.c_int32, C.c_void_p,
                                  C.c_void_p, C.c_int]
    L.j1_op_attention_noalloc.argtypes = L.j1_op_attention.argtypes
    L.j1_op_geglu_interleave.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]
    for fn in ("j1_config_load", "j1_model_create", "j1_model_config", "j1_model_forward", "j1_model_stage",
               "j1_model_launch", "j1_model_finish", "j1_engine_create", "j1_engine_create_pool",
               "j1_engine_logits_encoded", "j1_op_gemm", "j1_op_attention", "j1_op_attention_noalloc",
               "j1_op_geglu_interleave", "j1_model_profile", "j1_model_profile_read", "j1_encode_sequence",
               "j1_engine_logits_tokenized", "j1_router_create", "j1_router_create_with_scorer",
               "j1_router_route_many", "j1_tokenizer_load", "j1_tokenizer_from_json", "j1_tokenizer_encode",
               "j1_tokenizer_encode_batch", "j1_text_encoder_load", "j1_text_encoder_options",
               "j1_text_encoder_tokenize", "j1_text_encoder_encode"):
        getattr(L, fn).restype = C.c_int
    _lib = L
    return L


def last_error():
    buf = C.create_string_buffer(1024)
    lib().j1_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status):
    if status != OK:
        raise J1Error(status, last_error())


def _u32(a):
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a, a.ctypes.data_as(C.POINTER(C.c_uint32))


def _u8(a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a, a.ctypes.data_as(C.POINTER(C.c_uint8))


# ------------------------------------------------------------------ Device / options
@dataclass(frozen=True)
class Device:
    """Device::from_str (src/engine.rs:20-31): "cpu", "cuda", "cuda:N"."""
    kind: str
    index: int = 0

    @staticmethod
    def parse(s: str) -> "Device":
        if s == "cpu":
            return Device("cpu")
        if s == "cuda":
            return Device("cuda", 0)
        if s.startswith("cuda:") and s[5:].isdigit():
            return Device("cuda", int(s[5:]))
        raise J1Error(INVALID_ARG, "device must be cpu, cuda or cuda:N")

    def __str__(self):
        return "cpu" if self.kind == "cpu" else "cuda:%d" % self.index


@dataclass
class EngineOptions:
    """EngineOptions (src/engine.rs:34-65), device-side subset."""
    device: str = "cuda"
    batch_size: int = 16
    max_batch_tokens: int = 65536
    max_length: Optional[int] = None


def load_config(ckpt_dir):
    cfg = J1Config()
    check(lib().j1_config_load(ckpt_dir.encode(), C.byref(cfg)))
    return cfg


# ------------------------------------------------------------------ Batch / CudaModel
@dataclass
class Encoded:
    """encode::Encoded: token ids, marker positions within the row, question type."""
    ids: np.ndarray
    markers: np.ndarray
    qtype: int = 0


@dataclass
class Batch:
    """model::Batch (src/model.rs:225-269): sequences packed back to back, no padding."""
    ids: np.ndarray
    starts: np.ndarray
    lens: np.ndarray
    qtypes: np.ndarray
    marker_rows: np.ndarray
    marker_starts: np.ndarray

    @staticmethod
    def new(items: Sequence) -> "Batch":
        ids, starts, lens, qtypes, mrows, mstarts = [], [], [], [], [], [0]
        off = 0
        for it in items:
            e_ids, e_mk, e_qt = (it.ids, it.markers, it.qtype) if isinstance(it, Encoded) else it
            e_ids = np.asarray(e_ids, dtype=np.uint32)
            starts.append(off)
            lens.append(len(e_ids))
            qtypes.append(int(e_qt))
            ids.append(e_ids)
            mrows.extend(int(off + m) for m in np.asarray(e_mk).tolist())
            mstarts.append(len(mrows))
            off += len(e_ids)
        cat = np.concatenate(ids) if ids else np.zeros(0, np.uint32)
        return Batch(cat.astype(np.uint32), np.array(starts, np.uint32), np.array(lens, np.uint32),
                     np.array(qtypes, np.uint8), np.array(mrows, np.uint32), np.array(mstarts, np.uint32))

    def tokens(self):
        return int(self.ids.size)

    def split_scores(self, scores):
        return [list(map(float, scores[a:b])) for a, b in zip(self.marker_starts[:-1], self.marker_starts[1:])]


class CudaModel:
    """CudaModel (src/cuda/mod.rs:141-521) on one device, via libj1."""

    def __init__(self, ckpt_dir: str, ordinal: int = 0):
        h = C.c_void_p()
        check(lib().j1_model_create(ckpt_dir.encode(), int(ordinal), C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().j1_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def name(self):
        buf = C.create_string_buffer(256)
        lib().j1_model_name(self._h, buf, 256)
        return buf.value.decode()

    def config(self):
        cfg = J1Config()
        check(lib().j1_model_config(self._h, C.byref(cfg)))
        return cfg

    def _args(self, b: Batch):
        keep = [_u32(b.ids), _u32(b.starts), _u32(b.lens), _u8(b.qtypes), _u32(b.marker_rows), _u32(b.marker_starts)]
        p = [k[1] for k in keep]
        return keep, [p[0], b.ids.size, p[1], p[2], p[3], b.lens.size, p[4], p[5], b.marker_rows.size]

    def forward_flat(self, b: Batch) -> np.ndarray:
        keep, args = self._args(b)
        out = np.zeros(b.marker_rows.size, np.float32)
        check(lib().j1_model_forward(self._h, *args, out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def forward(self, b: Batch) -> List[List[float]]:
        """Scores per sequence (Batch::split_scores)."""
        return b.split_scores(self.forward_flat(b))

    def forward_many(self, batches: Sequence[Batch]) -> List[np.ndarray]:
        """j1_model_forward_many: the flat scores of each batch (pipelined staging)."""
        keep, jb, outs = [], (J1Batch * len(batches))(), []
        for i, b in enumerate(batches):
            k, a = self._args(b)
            keep.append(k)
            jb[i] = J1Batch(*a)
            outs.append(np.zeros(b.marker_rows.size, np.float32))
        po = (C.POINTER(C.c_float) * len(batches))(*[o.ctypes.data_as(C.POINTER(C.c_float)) for o in outs])
        check(lib().j1_model_forward_many(self._h, len(batches), jb, po))
        return outs

    # resident-batch split used by the benchmark
    def stage(self, b: Batch):
        self._staged = self._args(b)
        check(lib().j1_model_stage(self._h, *self._staged[1]))

    def launch(self):
        check(lib().j1_model_launch(self._h))

    def finish(self, m):
        out = np.zeros(m, np.float32)
        check(lib().j1_model_finish(self._h, out.ctypes.data_as(C.POINTER(C.c_float)), m))
        return out

    def stream(self):
        return lib().j1_model_stream(self._h)

    def launch_count(self):
        return int(lib().j1_model_launch_count(self._h))

    def profile(self, enable=True):
        """Per-launch CUDA-event timing by kernel family (j1_model_profile)."""
        check(lib().j1_model_profile(self._h, 1 if enable else 0))

    def profile_read(self):
        """{family: (total_ms, launches)} accumulated since profile(True)."""
        ms = (C.c_double * PROF_FAMILIES)()
        n = (C.c_int64 * PROF_FAMILIES)()
        check(lib().j1_model_profile_read(self._h, ms, n))
        return {lib().j1_profile_family_name(i).decode(): (ms[i], n[i]) for i in range(PROF_FAMILIES)}


# ------------------------------------------------------------------ Engine
class Engine:
    """Engine (src/engine.rs:73-284) restricted to the encoded-row API (no tokenizer)."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def load(ckpt_dir: str, options: Optional[EngineOptions] = None, devices: Optional[Sequence[int]] = None):
        o = options or EngineOptions()
        Device.parse(o.device)  # same parse errors as the reference
        copt = J1EngineOptions()
        lib().j1_engine_options_default(C.byref(copt))
        copt.device = o.device.encode()
        copt.batch_size = int(o.batch_size)
        copt.max_batch_tokens = int(o.max_batch_tokens)
        copt.max_length = int(o.max_length or 0)
        h = C.c_void_p()
        if devices:
            arr = (C.c_int * len(devices))(*devices)
            check(lib().j1_engine_create_pool(ckpt_dir.encode(), C.byref(copt), arr, len(devices), C.byref(h)))
        else:
            check(lib().j1_engine_create(ckpt_dir.encode(), C.byref(copt), C.byref(h)))
        return Engine(h)

    def close(self):
        if getattr(self, "_h", None):
            lib().j1_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_name(self):
        buf = C.create_string_buffer(1024)
        lib().j1_engine_device_name(self._h, buf, 1024)
        return buf.value.decode()

    def logits_encoded(self, rows: Sequence) -> List[List[float]]:
        """Raw option logits per row, in option order (Engine::logits_encoded)."""
        if len(rows) == 0:
            return []
        items = [r if isinstance(r, Encoded) else Encoded(*r) for r in rows]
        ids = np.concatenate([np.asarray(r.ids, np.uint32) for r in items])
        lens = np.array([len(r.ids) for r in items], np.uint32)
        mk = [np.asarray(r.markers, np.uint32) for r in items]
        markers = np.concatenate(mk) if mk else np.zeros(0, np.uint32)
        nmk = np.array([len(m) for m in mk], np.uint32)
        qt = np.array([int(r.qtype) for r in items], np.uint8)
        out = np.zeros(int(nmk.sum()), np.float32)
        keep = [_u32(ids), _u32(lens), _u32(markers), _u32(nmk), _u8(qt)]
        check(lib().j1_engine_logits_encoded(self._h, len(items), keep[0][1], keep[1][1], keep[2][1], keep[3][1],
                                             keep[4][1], out.ctypes.data_as(C.POINTER(C.c_float))))
        res, o = [], 0
        for n in nmk.tolist():
            res.append(list(map(float, out[o:o + n])))
            o += n
        return res

    def logits_flat(self, batch: "EncodedBatch") -> np.ndarray:
        """Engine::logits_encoded on an EncodedBatch (flat arrays, as TextEncoder.encode_batch
        returns with flat=True): all rows' option logits, row after row, as one float32 array."""
        n = int(batch.lens.size)
        out = np.zeros(int(batch.nmark.sum()), np.float32)
        if n == 0:
            return out
        keep = [_u32(batch.ids), _u32(batch.lens), _u32(batch.markers), _u32(batch.nmark), _u8(batch.qtypes)]
        check(lib().j1_engine_logits_encoded(self._h, n, keep[0][1], keep[1][1], keep[2][1], keep[3][1], keep[4][1],
                                             out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def logits_tokenized(self, rows: Sequence["TokenizedRequest"], enc: "EncoderOptions") -> List[List[float]]:
        """Engine::logits (src/engine.rs:236-243) on tokenized requests."""
        if len(rows) == 0:
            return []
        rq = _Requests(rows)
        o = enc.c()
        out = np.zeros(sum(len(r.options) for r in rows), np.float32)
        check(lib().j1_engine_logits_tokenized(self._h, C.byref(o), len(rows), rq.arr,
                                               out.ctypes.data_as(C.POINTER(C.c_float))))
        res, k = [], 0
        for r in rows:
            res.append(list(map(float, out[k:k + len(r.options)])))
            k += len(r.options)
        return res

    def logits(self, rows, text_encoder: "TextEncoder", threads: int = 0, flat: bool = False):
        """Engine::logits (src/engine.rs:236-243) on text requests (a list of Request, or a
        TextBatch): validate, encode in parallel on `threads` host threads (0 = all cores),
        logits_encoded. Per-row lists, or with flat=True one float32 array."""
        tb = rows if isinstance(rows, TextBatch) else TextBatch(rows)
        rows = tb.rows
        out = np.zeros(int(tb.n_options.sum()), np.float32)
        if tb.n == 0:
            return out if flat else []
        check(lib().j1_engine_logits_text(self._h, text_encoder._h, tb.n, tb.arr, int(threads or os.cpu_count() or 1),
                                          out.ctypes.data_as(C.POINTER(C.c_float))))
        if flat:
            return out
        res, k = [], 0
        for r in rows:
            res.append(list(map(float, out[k:k + len(r.options)])))
            k += len(r.options)
        return res

    def predict_encoded(self, rows, probabilities=False):
        """Engine::predict semantics on encoded rows: argmax index (+ softmax probabilities)."""
        out = []
        for z in self.logits_encoded(rows):
            z = np.asarray(z, np.float32)
            idx = int(np.argmax(z)) if z.size else 0
            pr = None
            if probabilities and z.size:
                e = np.exp((z - z.max()).astype(np.float64))
                pr = (e / e.sum()).tolist()
            out.append((idx, pr))
        return out


def plan_batches(row_lens, batch_size=16, max_batch_tokens=65536, n_devices=1):
    """The engine's micro-batch plan (j1_plan_batches): ([rows of batch b], [device of batch b])."""
    lens, lp = _u32(row_lens)
    n = lens.size
    bor = np.zeros(max(n, 1), np.uint32)
    dob = np.zeros(max(n, 1), np.uint32)
    nb = C.c_size_t()
    check(lib().j1_plan_batches(n, lp, int(batch_size), int(max_batch_tokens), int(n_devices),
                                bor.ctypes.data_as(C.POINTER(C.c_uint32)), dob.ctypes.data_as(C.POINTER(C.c_uint32)),
                                C.byref(nb)))
    batches = [[] for _ in range(nb.value)]
    for r in range(n):
        batches[int(bor[r])].append(r)
    # rows inside a batch keep the length-sorted order of the plan
    batches = [sorted(b, key=lambda r: (int(lens[r]), r)) for b in batches]
    return batches, [int(d) for d in dob[:nb.value]]


# ------------------------------------------------------------------ requests below the tokenizer, router
@dataclass
class EncoderOptions:
    """Encoder settings (src/encode.rs:25-38) without the tokenizer: special token ids and budgets.
    max_length 0 = the engine's max_length."""
    cls_id: int
    sep_id: int
    mask_id: int
    max_length: int = 0
    head_length: int = 256
    strict: bool = False

    def c(self):
        o = J1EncoderOptions()
        lib().j1_encoder_options_default(C.byref(o))
        o.cls_id, o.sep_id, o.mask_id = int(self.cls_id), int(self.sep_id), int(self.mask_id)
        o.max_length, o.head_length, o.strict = int(self.max_length), int(self.head_length), int(bool(self.strict))
        return o


@dataclass
class TokenizedRequest:
    """A Request (src/request.rs:77-82) after tokenization: tokens of
    "<qtype> question: <question>", of " <option>" per option, and of the rendered state."""
    head: Sequence[int]
    options: Sequence[Sequence[int]]
    state: Sequence[int]
    qtype: int = 0  # 0 choice, 1 score, 2 noul


class _Requests:
    """C views of a list of TokenizedRequest (keeps the arrays alive)."""

    def __init__(self, rows: Sequence[TokenizedRequest]):
        self.keep = []
        self.arr = (J1TokenizedRequest * max(len(rows), 1))()
        for i, r in enumerate(rows):
            head = np.ascontiguousarray(np.asarray(r.head, np.uint32).reshape(-1))
            state = np.ascontiguousarray(np.asarray(r.state, np.uint32).reshape(-1))
            opts = [np.asarray(x, np.uint32).reshape(-1) for x in r.options]
            oids = np.ascontiguousarray(np.concatenate(opts) if opts else np.zeros(0, np.uint32))
            olens = np.ascontiguousarray(np.array([x.size for x in opts], np.uint32))
            self.keep += [head, state, oids, olens]
            P = C.POINTER(C.c_uint32)
            self.arr[i] = J1TokenizedRequest(head.ctypes.data_as(P), head.size, oids.ctypes.data_as(P),
                                             olens.ctypes.data_as(P), len(opts), state.ctypes.data_as(P),
                                             state.size, int(r.qtype))


def encode_sequence(req: TokenizedRequest, opts: EncoderOptions):
    """Encoder::sequence (src/encode.rs:138-195) on ids -> (Encoded, truncated)."""
    o = opts.c()
    rq = _Requests([req])
    cap = max(int(o.max_length), 1)
    ids = np.zeros(cap, np.uint32)
    mk = np.zeros(max(len(req.options), 1), np.uint32)
    n, tr = C.c_size_t(), C.c_int32()
    check(lib().j1_encode_sequence(C.byref(o), rq.arr, ids.ctypes.data_as(C.POINTER(C.c_uint32)), cap, C.byref(n),
                                   mk.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(tr)))
    return Encoded(ids[:n.value].copy(), mk[:len(req.options)].copy(), int(req.qtype)), bool(tr.value)


def _check_text(rows: Sequence["Request"], line_prefix: bool):
    for i, r in enumerate(rows):
        if any(len(o) == 0 for o in r.options):
            raise J1Error(INVALID_ARG, ("JSONL line %d: options must contain 2–20 nonempty rendered descriptions"
                                        % (i + 1)) if line_prefix else "Options must be nonempty strings")




def display_probabilities(values: Sequence[float]) -> List[float]:
    """display_probabilities (src/request.rs:150-161)."""
    v = np.ascontiguousarray(np.asarray(values, np.float64))
    out = np.zeros(v.size, np.float64)
    lib().j1_display_probabilities(v.ctypes.data_as(C.POINTER(C.c_double)), v.size,
                                   out.ctypes.data_as(C.POINTER(C.c_double)))
    return out.tolist()


@dataclass
class RouteResult:
    """RouteResult (src/router.rs:15-26)."""
    index: int
    candidates: List[int]
    probabilities: List[float]
    rounds: int
    model_rows: int
    cache_hits: int
    hierarchical: bool
    probability_scope: str


class Router:
    """Router (src/router.rs) over an Engine, or over `scorer(rows) -> logits` where rows are
    Encoded (ids, markers, qtype) and logits one list of floats per row (e.g. a test double)."""

    def __init__(self, engine: Optional[Engine] = None, encoder: Optional[EncoderOptions] = None, scorer=None,
                 width=20, survivors=2, batch_size=16, cache_size=0, max_options=4096,
                 text_encoder: Optional["TextEncoder"] = None):
        self._text = text_encoder
        if encoder is None and text_encoder is not None:
            encoder = text_encoder.options()
        if encoder is None:
            raise J1Error(INVALID_ARG, "encoder options (special token ids) are required")
        ro = J1RouterOptions()
        lib().j1_router_options_default(C.byref(ro))
        ro.width, ro.survivors, ro.batch_size = int(width), int(survivors), int(batch_size)
        ro.cache_size, ro.max_options = int(cache_size), int(max_options)
        eo = encoder.c()
        h = C.c_void_p()
        self._engine, self._cb = engine, None
        if engine is not None:
            check(lib().j1_router_create(engine._h, C.byref(eo), C.byref(ro), C.byref(h)))
        elif scorer is not None:
            def cb(user, n, ids, lens, markers, nmark, qtypes, out):
                try:
                    ln = np.ctypeslib.as_array(lens, (n,)).copy()
                    nm = np.ctypeslib.as_array(nmark, (n,)).copy()
                    ii = np.ctypeslib.as_array(ids, (int(ln.sum()),)) if ln.sum() else np.zeros(0, np.uint32)
                    mm = np.ctypeslib.as_array(markers, (int(nm.sum()),)) if nm.sum() else np.zeros(0, np.uint32)
                    qq = np.ctypeslib.as_array(qtypes, (n,))
                    rows, t, k = [], 0, 0
                    for r in range(n):
                        rows.append(Encoded(ii[t:t + ln[r]].copy(), mm[k:k + nm[r]].copy(), int(qq[r])))
                        t += int(ln[r])
                        k += int(nm[r])
                    z = scorer(rows)
                    flat = np.concatenate([np.asarray(x, np.float32) for x in z]) if len(z) else np.zeros(0, np.float32)
                    if flat.size != int(nm.sum()):
                        return 2
                    dst = np.ctypeslib.as_array(out, (flat.size,)) if flat.size else None
                    if dst is not None:
                        dst[:] = flat
                    return 0
                except Exception:
                    return 1
            self._cb = SCORER_FN(cb)
            check(lib().j1_router_create_with_scorer(self._cb, None, C.byref(eo), C.byref(ro), C.byref(h)))
        else:
            raise J1Error(INVALID_ARG, "Router needs an engine or a scorer")
        self._h = h
        self.width, self.survivors, self.batch_size = int(width), int(survivors), int(batch_size)
        self.cache_size, self.max_options = int(cache_size), int(max_options)

    def close(self):
        if getattr(self, "_h", None):
            lib().j1_router_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clear_cache(self):
        lib().j1_router_clear_cache(self._h)

    @staticmethod
    def confident_winner(scores: Sequence[float], best: int) -> bool:
        """Router::confident_winner (src/router.rs:127-136)."""
        s = np.ascontiguousarray(np.asarray(scores, np.float32))
        return bool(lib().j1_router_confident_winner(s.ctypes.data_as(C.POINTER(C.c_float)), s.size, int(best)))

    def route_many(self, rows: Sequence) -> List[RouteResult]:
        """Router::route_many: batch independent groups across requests; request order kept.
        Rows are TokenizedRequest, or Request (text) when the router has a text_encoder."""
        if any(isinstance(r, Request) for r in rows):
            if self._text is None:
                raise J1Error(INVALID_ARG, "text requests need Router(text_encoder=...)")
            _check_text([r for r in rows if isinstance(r, Request)], False)
            rows = [self._text.tokenize_request(r) if isinstance(r, Request) else r for r in rows]
        rq = _Requests(rows)
        res = (J1RouteResult * max(len(rows), 1))()
        mr, ch = C.c_uint64(), C.c_uint64()
        check(lib().j1_router_route_many(self._h, len(rows), rq.arr, res, C.byref(mr), C.byref(ch)))
        out = []
        for i in range(len(rows)):
            r = res[i]
            n = int(r.n_candidates)
            hier = bool(r.hierarchical)
            out.append(RouteResult(int(r.index), [int(r.candidates[k]) for k in range(n)],
                                   [float(r.probabilities[k]) for k in range(n)], int(r.rounds), int(mr.value),
                                   int(ch.value), hier, "final_candidates" if hier else "all_options"))
        return out

    def route(self, row: TokenizedRequest) -> RouteResult:
        return self.route_many([row])[0]


# ------------------------------------------------------------------ text -> ids
QTYPES = {"choice": 0, "score": 1, "noul": 2}


class Tokenizer:
    """The checkpoint's tokenizer.json (byte-level BPE, HF `tokenizers` 0.22.2 format) in libj1:
    encode(text) == Tokenizer::encode_fast(text, false).ids (src/encode.rs:114-129)."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def from_file(path: str) -> "Tokenizer":
        h = C.c_void_p()
        check(lib().j1_tokenizer_load(path.encode(), C.byref(h)))
        return Tokenizer(h)

    @staticmethod
    def from_str(text: str) -> "Tokenizer":
        b = text.encode()
        h = C.c_void_p()
        check(lib().j1_tokenizer_from_json(b, len(b), C.byref(h)))
        return Tokenizer(h)

    def close(self):
        if getattr(self, "_h", None):
            lib().j1_tokenizer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def token_to_id(self, token: str) -> Optional[int]:
        v = lib().j1_tokenizer_token_to_id(self._h, token.encode())
        return None if v < 0 else int(v)

    def encode(self, text: str) -> List[int]:
        b = text.encode()
        cap = 4 * len(b) + 16
        out = np.zeros(cap, np.uint32)
        n = C.c_size_t()
        check(lib().j1_tokenizer_encode(self._h, b, len(b), out.ctypes.data_as(C.POINTER(C.c_uint32)), cap,
                                        C.byref(n)))
        return out[:n.value].tolist()

    def encode_batch(self, texts: Sequence[str], threads: int = 1, flat: bool = False):
        """Encode several texts on `threads` host threads. Returns a list of id lists, or with
        flat=True the (ids, offsets) arrays as the C ABI writes them."""
        bs = [t.encode() for t in texts]
        n = len(bs)
        if n == 0:
            return (np.zeros(0, np.uint32), np.zeros(1, np.uint64)) if flat else []
        mem, addr, blen = _cstrings(bs)
        addr, blen = np.ascontiguousarray(addr), np.ascontiguousarray(blen.astype(np.uint64))
        arr = addr.ctypes.data_as(C.POINTER(C.c_char_p))
        lens = blen.ctypes.data_as(C.POINTER(C.c_size_t))
        cap = int(blen.sum()) + n + 16
        ids = np.zeros(cap, np.uint32)
        offs = np.zeros(n + 1, np.uint64)
        check(lib().j1_tokenizer_encode_batch(self._h, n, arr, lens, int(threads),
                                              ids.ctypes.data_as(C.POINTER(C.c_uint32)), cap,
                                              offs.ctypes.data_as(C.POINTER(C.c_size_t))))
        if flat:
            return ids[:int(offs[-1])], offs
        return [ids[int(offs[i]):int(offs[i + 1])].tolist() for i in range(n)]


def inject_fault(kind: int, count: int = 1):
    """Host-side fault injection (j1_inject_fault): the next `count` device allocations
    (FAULT_ALLOC), kernel launches (FAULT_LAUNCH) or score readbacks (FAULT_NAN) fail; with
    FAULT_HOST the next entry points throw std::bad_alloc inside the library (-> OOM), with
    FAULT_WORKER the next host worker threads throw (-> INTERNAL); with FAULT_THREAD the next
    worker threads fail to start (the call finishes on the threads it has); with
    FAULT_DEVICE_WAIT the next op_attention_noalloc calls record a bounded device wait that
    timed out in their error word."""
    lib().j1_inject_fault(int(kind), int(count))


def selftest_device_timeout(ordinal: int = 0, limit_cycles: int = 2_000_000) -> int:
    """Bounded device wait on a barrier nothing arrives at; returns the status
    (DEVICE_TIMEOUT when the timeout was detected and reported)."""
    return int(lib().j1_selftest_device_timeout(int(ordinal), int(limit_cycles)))


def json_dumps(text: str) -> str:
    """State::render of a JSON state (src/pyjson.rs): json.dumps(value, ensure_ascii=False)
    of the JSON text, byte for byte."""
    b = text.encode()
    n = C.c_size_t()
    lib().j1_json_dumps(b, len(b), None, 0, C.byref(n))
    buf = C.create_string_buffer(n.value + 1)
    check(lib().j1_json_dumps(b, len(b), buf, n.value + 1, C.byref(n)))
    return buf.raw[:n.value].decode()


@dataclass
class Request:
    """request::Request (src/request.rs:77-82): `state` is the state text, or JSON text (an
    object or an array) with state_is_json=True, rendered like State::render."""
    state: str
    question: str
    options: Sequence[str]
    qtype: object = "choice"  # "choice" | "score" | "noul" or 0 | 1 | 2
    state_is_json: bool = False

    def qtype_id(self) -> int:
        return QTYPES[self.qtype] if isinstance(self.qtype, str) else int(self.qtype)


class TextBatch:
    """Text requests marshalled once for the C ABI (a j1_text_request array and the strings it
    points to), for calling several entry points on the same rows without rebuilding it."""

    def __init__(self, rows: Sequence["Request"]):
        self.rows = list(rows)
        self.n = len(self.rows)
        self.arr, self._keep = TextEncoder._text_rows(self.rows)
        rec = self._keep[2]
        self.n_options = rec["n_options"][:self.n].astype(np.int64)
        self.qtypes = rec["qtype"][:self.n].copy()


@dataclass
class EncodedBatch:
    """Encoded rows as flat arrays: ids of all rows back to back with their lengths, marker
    positions (within each row) with their counts per row, question types, truncation flags."""
    ids: np.ndarray
    lens: np.ndarray
    markers: np.ndarray
    nmark: np.ndarray
    qtypes: np.ndarray
    truncated: np.ndarray

    @staticmethod
    def empty() -> "EncodedBatch":
        z = np.zeros(0, np.uint32)
        return EncodedBatch(z, z, z, z, np.zeros(0, np.uint8), np.zeros(0, bool))

    def rows(self) -> List[Encoded]:
        i0 = np.concatenate([[0], np.cumsum(self.lens)]).astype(np.int64)
        m0 = np.concatenate([[0], np.cumsum(self.nmark)]).astype(np.int64)
        return [Encoded(self.ids[i0[k]:i0[k + 1]].copy(), self.markers[m0[k]:m0[k + 1]].copy(), int(self.qtypes[k]))
                for k in range(self.lens.size)]


class TextEncoder:
    """encode::Encoder (src/encode.rs:25-195) over the checkpoint's tokenizer: special tokens
    from tokenizer_config.json, LRU caches, the request's text forms and Encoder::sequence."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def load(ckpt_dir: str, max_length: int, head_length: int = 256, strict: bool = False,
             token_cache: int = 8192, encoding_cache: int = 2048) -> "TextEncoder":
        h = C.c_void_p()
        check(lib().j1_text_encoder_load(ckpt_dir.encode(), int(max_length), int(head_length), int(bool(strict)),
                                         int(token_cache), int(encoding_cache), C.byref(h)))
        return TextEncoder(h)

    def close(self):
        if getattr(self, "_h", None):
            lib().j1_text_encoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clear_cache(self):
        lib().j1_text_encoder_clear_cache(self._h)

    def options(self) -> EncoderOptions:
        o = J1EncoderOptions()
        check(lib().j1_text_encoder_options(self._h, C.byref(o)))
        return EncoderOptions(int(o.cls_id), int(o.sep_id), int(o.mask_id), int(o.max_length), int(o.head_length),
                              bool(o.strict))

    def tokenize(self, text: str) -> List[int]:
        b = text.encode()
        cap = 4 * len(b) + 16
        out = np.zeros(cap, np.uint32)
        n = C.c_size_t()
        check(lib().j1_text_encoder_tokenize(self._h, b, len(b), out.ctypes.data_as(C.POINTER(C.c_uint32)), cap,
                                             C.byref(n)))
        return out[:n.value].tolist()

    @staticmethod
    def _text_rows(rows: Sequence["Request"]):
        """The rows as a j1_text_request array (and what keeps its strings alive), built with
        numpy in a few passes rather than one ctypes object per string."""
        n = len(rows)
        nopt = np.fromiter((len(r.options) for r in rows), np.int64, n)
        strings = [r.state.encode() for r in rows] + [r.question.encode() for r in rows] + \
            [x.encode() for r in rows for x in r.options]
        mem, addr, _ = _cstrings(strings)
        optp = np.ascontiguousarray(addr[2 * n:]) if len(strings) > 2 * n else np.zeros(1, np.uint64)
        first = np.zeros(n, np.int64)
        if n > 1:
            np.cumsum(nopt[:-1], out=first[1:])
        rec = np.zeros(max(n, 1), _TEXT_DT)
        rec["state"][:n] = addr[:n]
        rec["question"][:n] = addr[n:2 * n]
        rec["options"][:n] = np.uint64(optp.ctypes.data) + (first * 8).astype(np.uint64)
        rec["n_options"][:n] = nopt
        rec["state_is_json"][:n] = np.fromiter((bool(r.state_is_json) for r in rows), np.int32, n)
        rec["qtype"][:n] = np.fromiter((r.qtype_id() for r in rows), np.uint8, n)
        return rec.ctypes.data_as(C.POINTER(J1TextRequest)), (mem, optp, rec)

    def encode_batch(self, rows, threads: int = 1, flat: bool = False):
        """Engine::encode's parallel Encoder::encode on a list of Request (or a TextBatch)
        -> [(Encoded, truncated)] in row order, or with flat=True one EncodedBatch."""
        tb = rows if isinstance(rows, TextBatch) else TextBatch(rows)
        rows, n, arr = tb.rows, tb.n, tb.arr
        if n == 0:
            return EncodedBatch.empty() if flat else []
        o = self.options()
        cap = n * o.max_length
        mcap = max(int(tb.n_options.sum()), 1)
        ids, mk = np.zeros(cap, np.uint32), np.zeros(mcap, np.uint32)
        offs, moffs, tr = np.zeros(n + 1, np.uint64), np.zeros(n + 1, np.uint64), np.zeros(n, np.int32)
        check(lib().j1_text_encoder_encode_batch(self._h, n, arr, int(threads),
                                                 ids.ctypes.data_as(C.POINTER(C.c_uint32)), cap,
                                                 offs.ctypes.data_as(C.POINTER(C.c_size_t)),
                                                 mk.ctypes.data_as(C.POINTER(C.c_uint32)), mcap,
                                                 moffs.ctypes.data_as(C.POINTER(C.c_size_t)),
                                                 tr.ctypes.data_as(C.POINTER(C.c_int32))))
        if flat:
            return EncodedBatch(ids[:int(offs[-1])], np.diff(offs).astype(np.uint32), mk[:int(moffs[-1])],
                                np.diff(moffs).astype(np.uint32), tb.qtypes.copy(), tr.astype(bool))
        return [(Encoded(ids[int(offs[i]):int(offs[i + 1])].copy(), mk[int(moffs[i]):int(moffs[i + 1])].copy(),
                         rows[i].qtype_id()), bool(tr[i])) for i in range(n)]

    def tokenize_request(self, r: "Request") -> TokenizedRequest:
        """The request's head, option and state tokens under Encoder::sequence's text rules."""
        q = r.qtype_id()
        opts = (C.c_char_p * max(len(r.options), 1))(*[x.encode() for x in r.options])
        total = C.c_size_t()
        L = lib()
        check(L.j1_text_encoder_request_tokens(self._h, r.state.encode(), r.question.encode(), opts, len(r.options),
                                               q, None, 0, C.byref(total), None))
        ids = np.zeros(max(total.value, 1), np.uint32)
        lens = np.zeros(len(r.options) + 2, np.uint32)
        check(L.j1_text_encoder_request_tokens(self._h, r.state.encode(), r.question.encode(), opts, len(r.options),
                                               q, ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size,
                                               C.byref(total), lens.ctypes.data_as(C.POINTER(C.c_uint32))))
        cut = np.concatenate([[0], np.cumsum(lens)]).astype(int)
        pieces = [ids[cut[i]:cut[i + 1]].tolist() for i in range(len(lens))]
        return TokenizedRequest(pieces[0], pieces[1:-1], pieces[-1], q)

    def encode(self, state: str, question: str, options: Sequence[str], qtype=0, state_is_json=False):
        """Encoder::encode on a request (state already rendered) -> (Encoded, truncated)."""
        q = QTYPES[qtype] if isinstance(qtype, str) else int(qtype)
        o = self.options()
        ids = np.zeros(o.max_length, np.uint32)
        mk = np.zeros(max(len(options), 1), np.uint32)
        opts = (C.c_char_p * max(len(options), 1))(*[x.encode() for x in options])
        n, tr = C.c_size_t(), C.c_int32()
        check(lib().j1_text_encoder_encode(self._h, state.encode(), int(bool(state_is_json)), question.encode(), opts,
                                           len(options), q, ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size,
                                           C.byref(n), mk.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(tr)))
        return Encoded(ids[:n.value].copy(), mk[:len(options)].copy(), q), bool(tr.value)


# ------------------------------------------------------------------ kernel-level ops (torch tensors)
def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def op_gemm(epilogue, A, W, out=None, bias=None, relu=False, x=None, ln_w=None, ln_b=None, ln_eps=1e-5, xn=None,
            pos=None, rope_cos=None, rope_sin=None, rope_cols=0, w2=None, b2=0.0, scores=None, stream=None, sync=True,
            grid_limit=0):
    """Fused-epilogue GEMM on torch CUDA tensors (bf16 A [M,K], W [N,K])."""
    M, K = A.shape
    N = W.shape[0]
    a = J1GemmArgs()
    a.epilogue, a.M, a.N, a.K = epilogue, M, N, K
    a.A, a.W = A.data_ptr(), W.data_ptr()
    a.out = out.data_ptr() if out is not None else None
    a.ldo = out.shape[1] if out is not None else 0
    a.bias = bias.data_ptr() if bias is not None else None
    a.relu = 1 if relu else 0
    a.x = x.data_ptr() if x is not None else None
    a.ldx = x.shape[1] if x is not None else 0
    a.ln_w = ln_w.data_ptr() if ln_w is not None else None
    a.ln_b = ln_b.data_ptr() if ln_b is not None else None
    a.ln_eps = ln_eps
    a.xn = xn.data_ptr() if xn is not None else None
    a.ldxn = xn.shape[1] if xn is not None else 0
    a.pos = pos.data_ptr() if pos is not None else None
    a.rope_cos = rope_cos.data_ptr() if rope_cos is not None else None
    a.rope_sin = rope_sin.data_ptr() if rope_sin is not None else None
    a.rope_cols = rope_cols
    a.w2 = w2.data_ptr() if w2 is not None else None
    a.b2 = b2
    a.scores = scores.data_ptr() if scores is not None else None
    a.grid_limit = grid_limit
    check(lib().j1_op_gemm(C.byref(a), C.c_void_p(stream) if stream else None, 1 if sync else 0))


def op_attention(qkv, hidden, seq_starts, seq_lens, window, ctx, stream=None, sync=True):
    s, sp = _u32(seq_starts)
    l, lp = _u32(seq_lens)
    check(lib().j1_op_attention(C.c_void_p(qkv.data_ptr()), qkv.shape[0], hidden, sp, lp, len(s), window,
                                C.c_void_p(ctx.data_ptr()), C.c_void_p(stream) if stream else None, 1 if sync else 0))


def op_attention_noalloc(qkv, hidden, seq_starts, seq_lens, window, ctx, stream=None, sync=True):
    """j1_op_attention_noalloc: op_attention with its scratch in a fixed device array."""
    s, sp = _u32(seq_starts)
    l, lp = _u32(seq_lens)
    check(lib().j1_op_attention_noalloc(C.c_void_p(qkv.data_ptr()), qkv.shape[0], hidden, sp, lp, len(s), window,
                                        C.c_void_p(ctx.data_ptr()), C.c_void_p(stream) if stream else None,
                                        1 if sync else 0))


def op_geglu_interleave(src_f32, dst_bf16, inter, k, stream=None):
    check(lib().j1_op_geglu_interleave(C.c_void_p(src_f32.data_ptr()), C.c_void_p(dst_bf16.data_ptr()), inter, k,
                                       C.c_void_p(stream) if stream else None))
