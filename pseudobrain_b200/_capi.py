"""ctypes binding of libpbk.so (include/pbk.h).

The library is the only compute path of this package: if it is missing or was
built for another ABI, importing this module raises, and nothing falls back to
PyTorch or to the CPU.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

PBK_ABI_VERSION = 1
PBK_OK = 0
PBK_ERR_INVALID, PBK_ERR_SHAPE, PBK_ERR_DTYPE, PBK_ERR_ALIGN = -1, -2, -3, -4
PBK_ERR_DEVICE, PBK_ERR_LAUNCH, PBK_ERR_WORKSPACE = -5, -6, -8
PBK_ERR_TIMEOUT = -7
PBK_IPC_HANDLE_BYTES = 64
PBK_ERR_TOO_LARGE = -9
PBK_QUEST_NOALLOC_MAX_SCORES = 4194304
PBK_F32, PBK_BF16 = 0, 1
PBK_STATE_KV, PBK_STATE_VK = 0, 1


class PbkView(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64), ("stride_t", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("dtype", ctypes.c_int32), ("pad_", ctypes.c_int32)]


class PbkDecodeExt(ctypes.Structure):
    _fields_ = [("gating", ctypes.c_int32), ("beta_round", ctypes.c_int32), ("softplus_beta", ctypes.c_float),
                ("softplus_threshold", ctypes.c_float), ("a", PbkView), ("b", PbkView), ("a_log", ctypes.c_void_p),
                ("dt_bias", ctypes.c_void_p), ("a_log_dtype", ctypes.c_int32), ("dt_bias_dtype", ctypes.c_int32),
                ("l2norm", ctypes.c_int32), ("eps", ctypes.c_float), ("null_slot", ctypes.c_int32),
                ("zero_skipped", ctypes.c_int32), ("cu_seqlens", ctypes.c_void_p), ("index_stride", ctypes.c_int64),
                ("num_accepted", ctypes.c_void_p)]


class PbkConvDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("hk", ctypes.c_int32), ("hv", ctypes.c_int32),
                ("width", ctypes.c_int32), ("l2mode", ctypes.c_int32), ("eps", ctypes.c_float), ("pad_", ctypes.c_int32),
                ("x", PbkView), ("tail", PbkView), ("new_tail", PbkView), ("weight", ctypes.c_void_p),
                ("q", PbkView), ("k", PbkView), ("v", PbkView)]


class PbkGatingDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("hv", ctypes.c_int32), ("pad_", ctypes.c_int32),
                ("decay", PbkView), ("a_log", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p),
                ("g", PbkView), ("beta", PbkView)]


class PbkOutNormDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("hv", ctypes.c_int32),
                ("weight_dtype", ctypes.c_int32), ("eps", ctypes.c_float), ("pad_", ctypes.c_int32),
                ("o", PbkView), ("gate", PbkView), ("out", PbkView), ("weight", ctypes.c_void_p)]


class PbkGdnLayerDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("hk", ctypes.c_int32), ("hv", ctypes.c_int32),
                ("width", ctypes.c_int32), ("l2mode", ctypes.c_int32), ("l2_eps", ctypes.c_float),
                ("norm_eps", ctypes.c_float), ("scale", ctypes.c_float), ("state_layout", ctypes.c_int32),
                ("qkv", PbkView), ("tail", PbkView), ("new_tail", PbkView), ("conv_weight", ctypes.c_void_p),
                ("decay", PbkView), ("a_log", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p), ("gate", PbkView),
                ("o_norm", ctypes.c_void_p), ("o_norm_dtype", ctypes.c_int32), ("pad_", ctypes.c_int32),
                ("out", PbkView), ("state", ctypes.c_void_p), ("state_slot_stride", ctypes.c_int64),
                ("state_indices", ctypes.c_void_p)]


class PbkTokenDesc(ctypes.Structure):
    _fields_ = [("t", ctypes.c_int32), ("h", ctypes.c_int32), ("kv", ctypes.c_int32), ("d", ctypes.c_int32),
                ("n_pool", ctypes.c_int32), ("full", ctypes.c_int32), ("hole_lo", ctypes.c_int32),
                ("hole_hi", ctypes.c_int32), ("rope_mask", ctypes.c_int32), ("block", ctypes.c_int32),
                ("q", ctypes.c_void_p), ("q_stride_t", ctypes.c_int64), ("q_stride_h", ctypes.c_int64),
                ("kmax", ctypes.c_void_p), ("kmin", ctypes.c_void_p), ("bnd_stride_kv", ctypes.c_int64),
                ("bnd_stride_p", ctypes.c_int64), ("keys", ctypes.c_void_p), ("key_stride_kv", ctypes.c_int64),
                ("key_stride_n", ctypes.c_int64), ("cand", ctypes.c_void_p), ("cand_stride_kv", ctypes.c_int64),
                ("out", ctypes.c_void_p), ("out_stride_kv", ctypes.c_int64), ("out_stride_t", ctypes.c_int64)]


class PbkGdnDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("hk", ctypes.c_int32),
                ("hv", ctypes.c_int32), ("dk", ctypes.c_int32), ("dv", ctypes.c_int32),
                ("q", PbkView), ("k", PbkView), ("v", PbkView), ("g", PbkView), ("beta", PbkView),
                ("o", PbkView), ("h0", ctypes.c_void_p), ("state", ctypes.c_void_p),
                ("state_slot_stride", ctypes.c_int64), ("state_layout", ctypes.c_int32),
                ("pad_", ctypes.c_int32), ("state_indices", ctypes.c_void_p), ("scale", ctypes.c_float),
                ("pad2_", ctypes.c_int32)]


class PbkQuestDesc(ctypes.Structure):
    _fields_ = [("nq", ctypes.c_int32), ("t", ctypes.c_int32), ("h", ctypes.c_int32), ("kv", ctypes.c_int32),
                ("d", ctypes.c_int32), ("page", ctypes.c_int32), ("n_arch", ctypes.c_int32),
                ("budget", ctypes.c_int32), ("n_win", ctypes.c_int32), ("window", ctypes.c_int32),
                ("sinks", ctypes.c_int32), ("scale", ctypes.c_float),
                ("q", ctypes.c_void_p), ("q_stride_n", ctypes.c_int64), ("q_stride_t", ctypes.c_int64),
                ("q_stride_h", ctypes.c_int64), ("qpos", ctypes.c_void_p),
                ("kmax", ctypes.c_void_p), ("kmin", ctypes.c_void_p), ("bnd_stride_kv", ctypes.c_int64),
                ("bnd_stride_p", ctypes.c_int64),
                ("keys", ctypes.c_void_p), ("values", ctypes.c_void_p), ("arc_stride_kv", ctypes.c_int64),
                ("arc_stride_n", ctypes.c_int64),
                ("win_keys", ctypes.c_void_p), ("win_values", ctypes.c_void_p), ("win_stride_kv", ctypes.c_int64),
                ("win_stride_n", ctypes.c_int64), ("kpos", ctypes.c_void_p),
                ("pages", ctypes.c_void_p), ("scores", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("out_stride_n", ctypes.c_int64), ("out_stride_t", ctypes.c_int64),
                ("out_stride_h", ctypes.c_int64), ("out_dtype", ctypes.c_int32), ("pad_", ctypes.c_int32)]


class PbkSwaDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("h", ctypes.c_int32), ("kv", ctypes.c_int32),
                ("d", ctypes.c_int32), ("window", ctypes.c_int32), ("sinks", ctypes.c_int32), ("scale", ctypes.c_float),
                ("q", PbkView), ("k", PbkView), ("v", PbkView), ("o", PbkView)]


class PbkQuestLevels(ctypes.Structure):
    _fields_ = [("smax", ctypes.c_void_p), ("smin", ctypes.c_void_p), ("sb_stride_kv", ctypes.c_int64),
                ("sb_stride_p", ctypes.c_int64), ("sblk", ctypes.c_int32), ("m_sb", ctypes.c_int32),
                ("hole_lo", ctypes.c_int32), ("hole_hi", ctypes.c_int32), ("pad_", ctypes.c_int32)]


class PbkRopeGatherDesc(ctypes.Structure):
    _fields_ = [("kv", ctypes.c_int32), ("d", ctypes.c_int32), ("block", ctypes.c_int32), ("n_blk", ctypes.c_int32),
                ("origin", ctypes.c_int32), ("n_rows", ctypes.c_int32), ("ref_pos", ctypes.c_int32),
                ("arc_span", ctypes.c_int32), ("mode", ctypes.c_int32), ("tail0", ctypes.c_int32),
                ("tail_n", ctypes.c_int32), ("scale", ctypes.c_float), ("const_delta", ctypes.c_float),
                ("pad_", ctypes.c_int32), ("blocks", ctypes.c_void_p), ("inv_freq", ctypes.c_void_p),
                ("keys", ctypes.c_void_p), ("values", ctypes.c_void_p), ("stride_kv", ctypes.c_int64),
                ("stride_n", ctypes.c_int64), ("out_keys", ctypes.c_void_p), ("out_values", ctypes.c_void_p),
                ("delta", ctypes.c_void_p)]


class PbkArchiveWriteDesc(ctypes.Structure):
    _fields_ = [("kv", ctypes.c_int32), ("d", ctypes.c_int32), ("block", ctypes.c_int32), ("origin", ctypes.c_int32),
                ("cap", ctypes.c_int32), ("size", ctypes.c_int32), ("p0", ctypes.c_int32), ("n", ctypes.c_int32),
                ("blk_lo", ctypes.c_int32), ("blk_hi", ctypes.c_int32), ("pos", ctypes.c_void_p),
                ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("in_stride_n", ctypes.c_int64),
                ("in_stride_kv", ctypes.c_int64), ("keys", ctypes.c_void_p), ("values", ctypes.c_void_p),
                ("arc_stride_kv", ctypes.c_int64), ("arc_stride_n", ctypes.c_int64), ("kmax", ctypes.c_void_p),
                ("kmin", ctypes.c_void_p), ("kmean", ctypes.c_void_p), ("vmean", ctypes.c_void_p),
                ("bnd_stride_kv", ctypes.c_int64), ("bnd_stride_p", ctypes.c_int64)]


_QD = ctypes.POINTER(PbkQuestDesc)
_QL = ctypes.POINTER(PbkQuestLevels)
_VP, _I32, _I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64

# name -> (restype, argtypes); every symbol include/pbk.h declares.
SIGNATURES = {
    "pbk_abi_version": (ctypes.c_int, []),
    "pbk_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "pbk_last_launch_error": (ctypes.c_char_p, []),
    "pbk_device_check": (ctypes.c_int, [ctypes.c_int]),
    "pbk_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "pbk_gdn_decode": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), ctypes.c_void_p]),
    "pbk_gdn_decode_ext": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), ctypes.POINTER(PbkDecodeExt),
                                          ctypes.c_void_p]),
    "pbk_gdn_prefill": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), ctypes.c_void_p]),
    "pbk_gdn_prefill_workspace": (ctypes.c_size_t, [ctypes.POINTER(PbkGdnDesc)]),
    "pbk_gdn_prefill_ws": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), _VP, ctypes.c_size_t, _VP]),
    "pbk_gdn_prefill_aux": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), ctypes.POINTER(PbkView),
                                           ctypes.POINTER(PbkView), _VP, ctypes.c_size_t, _VP]),
    "pbk_gdn_chunk_solve": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), _VP, ctypes.c_size_t, _VP]),
    "pbk_gdn_conv_norm": (ctypes.c_int, [ctypes.POINTER(PbkConvDesc), _VP]),
    "pbk_gdn_gating": (ctypes.c_int, [ctypes.POINTER(PbkGatingDesc), _VP]),
    "pbk_gdn_out_norm": (ctypes.c_int, [ctypes.POINTER(PbkOutNormDesc), _VP]),
    "pbk_gdn_decode_layer": (ctypes.c_int, [ctypes.POINTER(PbkGdnLayerDesc), _VP]),
    "pbk_gdn_prefill_layer_workspace": (ctypes.c_size_t, [ctypes.POINTER(PbkGdnLayerDesc)]),
    "pbk_gdn_prefill_layer": (ctypes.c_int, [ctypes.POINTER(PbkGdnLayerDesc), _VP, ctypes.c_size_t, _VP]),
    "pbk_gdn_prefill_varlen_workspace": (ctypes.c_size_t, [ctypes.POINTER(PbkGdnDesc), _I32]),
    "pbk_gdn_prefill_varlen": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), _VP, _I32, _VP, ctypes.c_size_t, _VP]),
    "pbk_gdn_prefill_solved": (ctypes.c_int, [ctypes.POINTER(PbkGdnDesc), _VP, ctypes.c_size_t, _VP]),
    "pbk_gdn_segment_scan": (ctypes.c_int, [_VP, _VP, _VP, _VP, _I32, _I32, _I32, _VP]),
    "pbk_quest_select_workspace": (ctypes.c_size_t, [_QD]),
    "pbk_quest_attend_workspace": (ctypes.c_size_t, [_QD]),
    "pbk_quest_select": (ctypes.c_int, [_QD, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_select_noalloc": (ctypes.c_int, [_QD, _VP]),
    "pbk_quest_select_parts": (ctypes.c_int, [_QD, _I32, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_attend_parts": (ctypes.c_int, [_QD, _VP, _VP, _I32, _I64, _I64, _I32, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_attend": (ctypes.c_int, [_QD, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_attend_sinks_workspace": (ctypes.c_size_t, [_QD, _I32]),
    "pbk_quest_attend_sinks": (ctypes.c_int, [_QD, _VP, _VP, _I32, _I64, _I64, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_rerank_workspace": (ctypes.c_size_t, [_QD, _I32]),
    "pbk_quest_rerank": (ctypes.c_int, [_QD, _VP, _I32, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_gather": (ctypes.c_int, [_QD, _I32, _VP, _VP, _VP]),
    "pbk_quest_bounds": (ctypes.c_int, [_VP, _I32, _I32, _I32, _I32, _I64, _I64, _VP, _VP, _I64, _I64, _I32, _VP]),
    "pbk_quest_superbounds": (ctypes.c_int, [_VP, _VP, _I32, _I32, _I32, _I32, _I64, _I64, _VP, _VP, _I64, _I64,
                                             _I32, _I32, _VP]),
    "pbk_quest_select_levels_workspace": (ctypes.c_size_t, [_QD, _QL]),
    "pbk_quest_select_levels": (ctypes.c_int, [_QD, _QL, _VP, ctypes.c_size_t, _VP]),
    "pbk_quest_rope_gather": (ctypes.c_int, [ctypes.POINTER(PbkRopeGatherDesc), _VP]),
    "pbk_quest_archive_write": (ctypes.c_int, [ctypes.POINTER(PbkArchiveWriteDesc), _VP]),
    "pbk_quest_supermeans": (ctypes.c_int, [_VP, _I32, _I32, _I32, _I32, _I64, _I64, _VP, _I64, _I64, _I32, _I32,
                                            _VP]),
    "pbk_l2norm": (ctypes.c_int, [PbkView, PbkView, _I32, _I32, _I32, _I32, ctypes.c_float, _VP]),
    "pbk_swa_prefill": (ctypes.c_int, [ctypes.POINTER(PbkSwaDesc), _VP]),
    "pbk_quest_token_scores": (ctypes.c_int, [ctypes.POINTER(PbkTokenDesc), _VP]),
    "pbk_quest_token_rerank": (ctypes.c_int, [ctypes.POINTER(PbkTokenDesc), _VP]),
    "pbk_quest_row_ranks": (ctypes.c_int, [_VP, _I64, _I32, _I32, _VP, _I64, _VP]),
    "pbk_ipc_handle": (ctypes.c_int, [_VP, _VP, ctypes.POINTER(ctypes.c_int64)]),
    "pbk_ipc_open": (ctypes.c_int, [_VP, ctypes.POINTER(ctypes.c_void_p)]),
    "pbk_ipc_close": (ctypes.c_int, [_VP]),
    "pbk_copy_async": (ctypes.c_int, [_VP, _VP, ctypes.c_size_t, _VP]),
}


def _load() -> ctypes.CDLL:
    path = _build.LIB_PATH
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m pseudobrain_b200.build` "
                          "(this package has no CPU or PyTorch fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    if lib.pbk_abi_version() != PBK_ABI_VERSION:
        raise ImportError(f"{path} has ABI {lib.pbk_abi_version()}, expected {PBK_ABI_VERSION}: rebuild it")
    return lib


LIB = _load()


class PbkError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = f"{what}: {LIB.pbk_status_string(status).decode()} (status {status})"
        if status == -6:
            msg += f": {LIB.pbk_last_launch_error().decode()}"
        super().__init__(msg)


def check(status: int, what: str) -> None:
    if status != PBK_OK:
        raise PbkError(status, what)


def device_error(clear: bool = True) -> int:
    """The current device's error word (nonzero: a tensor-core kernel's bounded wait gave
    up; the code names the wait site). Synchronises with the device."""
    code = ctypes.c_int(0)
    check(LIB.pbk_device_error(ctypes.byref(code), int(clear)), "pbk_device_error")
    return code.value
