"""Python bindings (ctypes) for the kim-kvcache B200 library.

The product is the shared library lib/libkk_b200.so: the C++ host token-loop
runtime and the sm_100a CUDA kernels behind the C ABI declared in
include/kk_runtime.h and include/kk_kernels.h. This module only loads that
library and describes its C signatures; it contains no compute of its own.
It raises ImportError-style errors when the library is missing instead of
falling back to anything else.

The directory name is not a valid Python identifier, so callers load it by
path, e.g. ``kk = load_package()`` from the repository root helper below.
"""
from __future__ import annotations

import ctypes as C
import importlib.util
import os
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libkk_b200.so"


class KkEntry(C.Structure):
    _fields_ = [("logical_token_begin", C.c_uint32), ("valid_tokens", C.c_uint16),
                ("kind", C.c_uint8), ("reserved", C.c_uint8), ("slot", C.c_uint32),
                ("generation", C.c_uint32)]


class KkHandle(C.Structure):
    _fields_ = [("kind", C.c_uint8), ("reserved", C.c_uint8 * 3), ("slot", C.c_uint32),
                ("generation", C.c_uint32)]


class KkPageMeta(C.Structure):
    _fields_ = [("state", C.c_uint8), ("reserved", C.c_uint8), ("valid_tokens", C.c_uint16),
                ("ref_count", C.c_uint32), ("promotion_pins", C.c_uint32),
                ("inflight_readers", C.c_uint32), ("mutable_owner", C.c_uint64)]


class KkPoolSnapshot(C.Structure):
    _fields_ = [("total_slots", C.c_uint32), ("free_slots", C.c_uint32),
                ("allocated_slots", C.c_uint32), ("reserved", C.c_uint32),
                ("successful_allocations", C.c_uint64), ("successful_releases", C.c_uint64),
                ("failed_allocations", C.c_uint64), ("rejected_releases", C.c_uint64)]


class KkMgrSnapshot(C.Structure):
    _fields_ = [("request_count", C.c_uint64), ("promotion_count", C.c_uint64),
                ("page_lease_count", C.c_uint64), ("token_reservation_count", C.c_uint64),
                ("micro_pool", KkPoolSnapshot), ("extent_pool", KkPoolSnapshot)]


class KkFixedSnapshot(C.Structure):
    _fields_ = [("request_count", C.c_uint64), ("successful_allocations", C.c_uint64),
                ("peak_allocated_pages", C.c_uint64), ("token_reservation_count", C.c_uint64),
                ("pool", KkPoolSnapshot)]


class KkTableOut(C.Structure):
    _fields_ = [("entries", C.POINTER(KkEntry)), ("capacity", C.c_uint32),
                ("count", C.c_uint32), ("version", C.c_uint64)]


def _struct_tuple(s: C.Structure) -> tuple:
    out = []
    for name, _ in s._fields_:
        if name == "reserved":
            continue
        v = getattr(s, name)
        out.append(_struct_tuple(v) if isinstance(v, C.Structure) else v)
    return tuple(out)


_P = C.c_void_p
_U32, _U64, _I = C.c_uint32, C.c_uint64, C.c_int
MANAGER_SIGNATURES = {
    "mgr_create": (_P, [_U32, _U32]),
    "mgr_destroy": (None, [_P]),
    "mgr_create_request": (_I, [_P, _U64]),
    "mgr_append": (_I, [_P, _U64, _U32]),
    "mgr_reserve_token": (_I, [_P, _U64, _U32, C.POINTER(_U64), C.POINTER(KkTableOut),
                               C.POINTER(KkTableOut)]),
    "mgr_commit_reservation": (_I, [_P, _U64]),
    "mgr_rollback_reservation": (_I, [_P, _U64]),
    "mgr_seal_tail": (_I, [_P, _U64]),
    "mgr_fork": (_I, [_P, _U64, _U64]),
    "mgr_release": (_I, [_P, _U64]),
    "mgr_prepare_promotion": (_I, [_P, _U64, _U32, C.POINTER(_U64), C.POINTER(KkHandle),
                                   C.POINTER(KkHandle)]),
    "mgr_commit_promotion": (_I, [_P, _U64]),
    "mgr_rollback_promotion": (_I, [_P, _U64]),
    "mgr_acquire_request_lease": (_I, [_P, _U64, C.POINTER(_U64), C.POINTER(_U32)]),
    "mgr_acquire_promotion_lease": (_I, [_P, _U64, C.POINTER(_U64), C.POINTER(_U32)]),
    "mgr_acquire_reservation_lease": (_I, [_P, _U64, C.POINTER(_U64), C.POINTER(_U32)]),
    "mgr_release_lease": (_I, [_P, _U64]),
    "mgr_block_table": (_I, [_P, _U64, C.POINTER(KkTableOut)]),
    "mgr_page_metadata": (_I, [_P, KkHandle, C.POINTER(KkPageMeta)]),
    "mgr_snapshot": (None, [_P, C.POINTER(KkMgrSnapshot)]),
    "mgr_check_invariants": (_I, [_P]),
    "float_to_half": (C.c_uint16, [C.c_float]),
    "half_to_float": (C.c_float, [C.c_uint16]),
}


FIXED_SIGNATURES = {
    "fixed_create": (_P, [C.c_uint16, _U32]),
    "fixed_destroy": (None, [_P]),
    "fixed_tokens_per_page": (_U32, [_P]),
    "fixed_create_request": (_I, [_P, _U64]),
    "fixed_append": (_I, [_P, _U64, _U32]),
    "fixed_reserve_token": (_I, [_P, _U64, _U32, C.POINTER(_U64), C.POINTER(KkTableOut),
                                 C.POINTER(KkTableOut)]),
    "fixed_commit_reservation": (_I, [_P, _U64]),
    "fixed_rollback_reservation": (_I, [_P, _U64]),
    "fixed_seal_tail": (_I, [_P, _U64]),
    "fixed_fork": (_I, [_P, _U64, _U64]),
    "fixed_release": (_I, [_P, _U64]),
    "fixed_block_table": (_I, [_P, _U64, C.POINTER(KkTableOut)]),
    "fixed_snapshot": (None, [_P, C.POINTER(KkFixedSnapshot)]),
    "fixed_check_invariants": (_I, [_P]),
}


def bind(lib: C.CDLL, prefix: str, signatures: dict) -> dict:
    """Attaches argtypes/restype to every `prefix + name` symbol; returns name->fn."""
    fns = {}
    for name, (res, args) in signatures.items():
        fn = getattr(lib, prefix + name)
        fn.restype = res
        fn.argtypes = args
        fns[name] = fn
    return fns


_LIB = None


def load_library() -> C.CDLL:
    """Loads lib/libkk_b200.so (built by build.py). Raises OSError if absent."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} is missing: run `python kim-kvcache_b200/build.py`")
        _LIB = C.CDLL(str(LIB_PATH))
    return _LIB


class Manager:
    """KvCacheManager through a C ABI (`prefix` kkrt_ = this library, kref_ =
    the reference oracle twin with identical signatures)."""

    MAX_ENTRIES = 4096

    def __init__(self, lib: C.CDLL, prefix: str, micro: int, extent: int):
        self.f = bind(lib, prefix, MANAGER_SIGNATURES)
        self.h = self.f["mgr_create"](micro, extent)
        if not self.h:
            raise ValueError("invalid capacities")
        self._buf = [(KkEntry * self.MAX_ENTRIES)() for _ in range(2)]

    def close(self):
        if self.h:
            self.f["mgr_destroy"](self.h)
            self.h = None

    __del__ = close

    def _table(self, i=0):
        return KkTableOut(C.cast(self._buf[i], C.POINTER(KkEntry)), self.MAX_ENTRIES, 0, 0)

    @staticmethod
    def _entries(t: KkTableOut, buf) -> tuple:
        return (t.version, tuple(_struct_tuple(buf[i]) for i in range(t.count)))

    def create(self, rid):
        return self.f["mgr_create_request"](self.h, rid)

    def append(self, rid, n):
        return self.f["mgr_append"](self.h, rid, n)

    def reserve(self, rid, expected):
        r = C.c_uint64(0)
        b, v = self._table(0), self._table(1)
        err = self.f["mgr_reserve_token"](self.h, rid, expected, C.byref(r), C.byref(b), C.byref(v))
        return err, r.value, self._entries(b, self._buf[0]), self._entries(v, self._buf[1])

    def commit(self, res_id):
        return self.f["mgr_commit_reservation"](self.h, res_id)

    def rollback(self, res_id):
        return self.f["mgr_rollback_reservation"](self.h, res_id)

    def seal(self, rid):
        return self.f["mgr_seal_tail"](self.h, rid)

    def fork(self, src, child):
        return self.f["mgr_fork"](self.h, src, child)

    def release(self, rid):
        return self.f["mgr_release"](self.h, rid)

    def prepare_promotion(self, rid, begin):
        pid = C.c_uint64(0)
        src = (KkHandle * 8)()
        tgt = KkHandle()
        err = self.f["mgr_prepare_promotion"](self.h, rid, begin, C.byref(pid), src, C.byref(tgt))
        return err, pid.value, tuple(_struct_tuple(s) for s in src), _struct_tuple(tgt)

    def commit_promotion(self, pid):
        return self.f["mgr_commit_promotion"](self.h, pid)

    def rollback_promotion(self, pid):
        return self.f["mgr_rollback_promotion"](self.h, pid)

    def _lease(self, name, key):
        lid, n = C.c_uint64(0), C.c_uint32(0)
        err = self.f[name](self.h, key, C.byref(lid), C.byref(n))
        return err, lid.value, n.value

    def lease_request(self, rid):
        return self._lease("mgr_acquire_request_lease", rid)

    def lease_promotion(self, pid):
        return self._lease("mgr_acquire_promotion_lease", pid)

    def lease_reservation(self, res_id):
        return self._lease("mgr_acquire_reservation_lease", res_id)

    def release_lease(self, lid):
        return self.f["mgr_release_lease"](self.h, lid)

    def table(self, rid):
        t = self._table(0)
        if not self.f["mgr_block_table"](self.h, rid, C.byref(t)):
            return None
        return self._entries(t, self._buf[0])

    def page_meta(self, kind, slot, generation):
        m = KkPageMeta()
        h = KkHandle(kind, (C.c_uint8 * 3)(), slot, generation)
        if not self.f["mgr_page_metadata"](self.h, h, C.byref(m)):
            return None
        return _struct_tuple(m)

    def snapshot(self):
        s = KkMgrSnapshot()
        self.f["mgr_snapshot"](self.h, C.byref(s))
        return _struct_tuple(s)

    def invariants(self):
        return bool(self.f["mgr_check_invariants"](self.h))


class FixedManager:
    """FixedPageManager through a C ABI (kkrt_ = this library, kref_ = the
    reference oracle twin). Same method names and result tuples as Manager."""

    MAX_ENTRIES = 4096

    def __init__(self, lib: C.CDLL, prefix: str, tokens_per_page: int, capacity: int):
        self.f = bind(lib, prefix, FIXED_SIGNATURES)
        self.h = self.f["fixed_create"](tokens_per_page, capacity)
        if not self.h:
            raise ValueError("invalid page size or capacity")
        self._buf = [(KkEntry * self.MAX_ENTRIES)() for _ in range(2)]

    def close(self):
        if self.h:
            self.f["fixed_destroy"](self.h)
            self.h = None

    __del__ = close

    def _table(self, i=0):
        return KkTableOut(C.cast(self._buf[i], C.POINTER(KkEntry)), self.MAX_ENTRIES, 0, 0)

    def tokens_per_page(self):
        return self.f["fixed_tokens_per_page"](self.h)

    def create(self, rid):
        return self.f["fixed_create_request"](self.h, rid)

    def append(self, rid, n):
        return self.f["fixed_append"](self.h, rid, n)

    def reserve(self, rid, expected):
        r = C.c_uint64(0)
        b, v = self._table(0), self._table(1)
        err = self.f["fixed_reserve_token"](self.h, rid, expected, C.byref(r), C.byref(b), C.byref(v))
        return err, r.value, Manager._entries(b, self._buf[0]), Manager._entries(v, self._buf[1])

    def commit(self, res_id):
        return self.f["fixed_commit_reservation"](self.h, res_id)

    def rollback(self, res_id):
        return self.f["fixed_rollback_reservation"](self.h, res_id)

    def seal(self, rid):
        return self.f["fixed_seal_tail"](self.h, rid)

    def fork(self, src, child):
        return self.f["fixed_fork"](self.h, src, child)

    def release(self, rid):
        return self.f["fixed_release"](self.h, rid)

    def table(self, rid):
        t = self._table(0)
        if not self.f["fixed_block_table"](self.h, rid, C.byref(t)):
            return None
        return Manager._entries(t, self._buf[0])

    def snapshot(self):
        s = KkFixedSnapshot()
        self.f["fixed_snapshot"](self.h, C.byref(s))
        return _struct_tuple(s)

    def invariants(self):
        return bool(self.f["fixed_check_invariants"](self.h))


# ---- kernel C ABI (include/kk_kernels.h) ------------------------------------

KK_EINVAL = 1000
KK_ENOSCRATCH = 1001
ATTN_SCRATCH_BYTES = 4 << 20
ATTN_AUTO, ATTN_DIRECT, ATTN_TMA = 0, 1, 2
ATTN_ITEM_MULTI_LANE = 1
W_ROW_MAJOR, W_PACKED = 0, 1
EPI_STORE_F16, EPI_STORE_F32, EPI_RESIDUAL, EPI_SILU_PAIRS, EPI_QKV_ROPE, EPI_ARGMAX = range(6)


class KvPools(C.Structure):
    _fields_ = [("micro", C.c_void_p), ("extent", C.c_void_p), ("micro_capacity", C.c_uint32),
                ("extent_capacity", C.c_uint32), ("layers", C.c_uint32), ("kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("micro_page_tokens", C.c_uint32)]


class PageDesc(C.Structure):
    _fields_ = [("slot", C.c_uint32), ("logical_token_begin", C.c_uint32),
                ("valid_tokens", C.c_uint16), ("kind", C.c_uint8), ("reserved0", C.c_uint8),
                ("reserved1", C.c_uint32)]


class KvSlot(C.Structure):
    _fields_ = [("slot", C.c_uint32), ("page_token", C.c_uint16), ("kind", C.c_uint8),
                ("active", C.c_uint8)]


class KvCopy(C.Structure):
    _fields_ = [("src_slot", C.c_uint32), ("dst_slot", C.c_uint32), ("tokens", C.c_uint16),
                ("src_kind", C.c_uint8), ("dst_kind", C.c_uint8)]


class AttnLane(C.Structure):
    _fields_ = [("desc_offset", C.c_uint32), ("desc_count", C.c_uint32),
                ("token_count", C.c_uint32), ("item_offset", C.c_uint32),
                ("item_count", C.c_uint32), ("query_row", C.c_uint32),
                ("first_item_shared", C.c_uint32), ("reserved", C.c_uint32)]


class AttnItem(C.Structure):
    _fields_ = [("lane", C.c_uint32), ("desc_begin", C.c_uint32), ("desc_end", C.c_uint32),
                ("reserved", C.c_uint32)]


class GemmDesc(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("M", C.c_uint32), ("K", C.c_uint32), ("x", C.c_void_p),
                ("N", C.c_uint32), ("x_stride", C.c_uint32), ("x_rows", C.c_uint32),
                ("epilogue", C.c_uint32), ("out", C.c_void_p), ("out_stride", C.c_uint32),
                ("split_k", C.c_uint32), ("positions", C.c_void_p), ("slots", C.c_void_p),
                ("pools", KvPools), ("layer", C.c_uint32), ("q_rows", C.c_uint32),
                ("kv_rows", C.c_uint32), ("head_dim", C.c_uint32), ("rope_theta", C.c_float),
                ("tokens", C.c_void_p), ("argmax_workspace", C.c_void_p),
                ("weight_layout", C.c_uint32), ("norm_input", C.c_void_p),
                ("norm_stride", C.c_uint32), ("norm_eps", C.c_float), ("norm_weight", C.c_void_p),
                ("rope_cos_sin", C.c_void_p), ("rope_positions", C.c_uint32)]


_VP = C.c_void_p
KERNEL_SIGNATURES = {
    "attention_plan": (_U32, [C.POINTER(PageDesc), C.POINTER(AttnLane), _U32, _U32,
                              C.POINTER(AttnItem), _U32]),
    "paged_decode_attention_noalloc": (_I, [C.POINTER(KvPools), _U32, _U32, _VP, _VP, _U32, _VP,
                                            _U32, _VP, _U32, _VP, _U32, C.c_float, _VP]),
    "attention_plan_balanced": (_U32, [C.POINTER(PageDesc), C.POINTER(AttnLane), _U32, _U32,
                                       C.POINTER(AttnItem), _U32]),
    "attention_workspace_bytes": (_U64, [_U32, _U32, _U32, _U32]),
    "attention_workspace_init": (_I, [_VP, _U32, _VP]),
    "paged_decode_attention": (_I, [C.POINTER(KvPools), _U32, _U32, _VP, _VP, _U32, _VP, _U32,
                                    _VP, _U32, _VP, _U32, C.c_float, _VP, _U64, _VP]),
    "kv_write": (_I, [C.POINTER(KvPools), _U32, _U32, _VP, _U32, _VP, _VP, _U64, _U64, _VP]),
    "kv_copy_tokens": (_I, [C.POINTER(KvPools), _U32, _U32, _VP, _U32, _VP]),
    "rmsnorm": (_I, [_VP, _VP, _VP, _U32, _U32, C.c_float, _VP]),
    "embed_rmsnorm": (_I, [_VP, _VP, _VP, _VP, _VP, _U32, _U32, C.c_float, _VP]),
    "rope": (_I, [_VP, _U32, _VP, _U32, _VP, _U32, _U32, _U32, _U32, C.c_float, _VP]),
    "silu_mul": (_I, [_VP, _VP, _VP, _U32, _U32, _VP]),
    "residual_add": (_I, [_VP, _VP, _U64, _VP]),
    "argmax_workspace_bytes": (_U64, [_U32, _U32]),
    "gemm": (_I, [C.POINTER(GemmDesc), _VP]),
    "gemm_packed_bytes": (_U64, [_U32, _U32]),
    "gemm_pack_weight": (_I, [_VP, _U32, _U32, _VP, _VP]),
    "gemm_pack_weight_scaled": (_I, [_VP, _U32, _U32, _VP, _VP, _VP]),
    "kv_promote": (_I, [C.POINTER(KvPools), C.POINTER(_U32), _U32, _VP]),
    "kv_gather": (_I, [C.POINTER(KvPools), _VP, _U32, _U32, _VP, _VP]),
    "kv_scatter": (_I, [C.POINTER(KvPools), _VP, _U32, _U32, _U32, _VP, _VP]),
    "fill_fp16": (_I, [_VP, _U64, _U64, C.c_float, _VP]),
    "device_status": (_I, [_VP]),
    "debug_attention_fault": (_I, [_U32, _U64]),
    "set_pdl": (None, [_I]),
    "attention_set_variant": (_I, [_I]),
}

_KERNELS = None


def kernels() -> dict:
    """name -> ctypes function for every kk_* kernel entry point."""
    global _KERNELS
    if _KERNELS is None:
        _KERNELS = bind(load_library(), "kk_", KERNEL_SIGNATURES)
    return _KERNELS


# ---- runtime C ABI (include/kk_runtime.h): backend, transactions, runner, scheduler ----

class BackendSnapshot(C.Structure):
    _fields_ = [("request_count", C.c_uint64), ("active_transaction_count", C.c_uint64),
                ("committed_token_count", C.c_uint64), ("batched_attention_submissions", C.c_uint64),
                ("batched_attention_lanes", C.c_uint64), ("allocated_micro_pages", C.c_uint32),
                ("allocated_extent_pages", C.c_uint32), ("storage_reserved_bytes", C.c_uint64)]


class Terminal(C.Structure):
    _fields_ = [("request_id", C.c_uint64), ("reason", C.c_uint8), ("error", C.c_uint8),
                ("reserved", C.c_uint16), ("token_count", C.c_uint32),
                ("prompt_tokens", C.c_uint32), ("completion_tokens", C.c_uint32),
                ("ttft_ns", C.c_uint64), ("tpot_ns", C.c_uint64), ("e2e_ns", C.c_uint64)]


class Iteration(C.Structure):
    _fields_ = [("iteration", C.c_uint64), ("model_forward_tokens", C.c_uint32),
                ("model_forward_batches", C.c_uint32), ("prefill_tokens", C.c_uint32),
                ("decode_tokens", C.c_uint32), ("terminals_produced", C.c_uint32),
                ("reserved", C.c_uint32)]


_I64, _F = C.c_int64, C.c_float
_PU32, _PU64 = C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)
RUNTIME_SIGNATURES = {
    "backend_create": (_VP, [_U32, _U32, _U32, _U32, _U64, _U32, _U32]),
    "fixed_backend_create": (_VP, [_U32, _U32, _U32, _U32, _U64, _U32, _U32]),
    "backend_kind": (_I, [_VP]),
    "backend_destroy": (None, [_VP]),
    "backend_create_request": (_I, [_VP, _U64]),
    "backend_fork": (_I, [_VP, _U64, _U64]),
    "backend_release": (_I, [_VP, _U64]),
    "backend_check_invariants": (_I, [_VP]),
    "backend_snapshot": (None, [_VP, C.POINTER(BackendSnapshot)]),
    "backend_inject_failure": (_I, [_VP, _I]),
    "backend_pools": (_I, [_VP, C.POINTER(KvPools)]),
    "backend_block_table": (_I, [_VP, _U64, C.POINTER(KkTableOut)]),
    "backend_append": (_I, [_VP, _U64, _U32]),
    "backend_seal": (_I, [_VP, _U64]),
    "backend_promote": (_I, [_VP, _U64, _U32, _VP]),
    "backend_gather": (_I, [_VP, _U64, _VP, _VP]),
    "txn_reserve": (_VP, [_VP, _U64, _U32, _VP, C.POINTER(_I)]),
    "txn_write_layer": (_I, [_VP, _U32, _VP, _VP]),
    "txn_attend_layer": (_I, [_VP, _U32, _VP, _VP, _VP, _U64, _F]),
    "txn_attend_batch": (None, [C.POINTER(_VP), _U32, _U32, _VP, _VP, _U64, _VP, _U64, _F,
                                C.POINTER(_I)]),
    "txn_reserved_table": (_I, [_VP, C.POINTER(KkTableOut)]),
    "txn_commit": (_I, [_VP]),
    "txn_rollback": (_I, [_VP]),
    "txn_phase": (_I, [_VP]),
    "txn_destroy": (None, [_VP]),
    "runner_create": (_VP, [C.c_char_p, C.c_char_p, _VP, _VP, _U32, _I, _I, C.POINTER(_I),
                            C.c_char_p, _U32]),
    "runner_destroy": (None, [_VP]),
    "runner_set_auto_promote": (_I, [_VP, _I]),
    "runner_prefill": (_I, [_VP, C.c_uint64, _PU32, _U32, _U32, _PU32]),
    "runner_forward_batch": (_I, [_VP, _U32, _PU64, _PU32, _PU32, _PU32, C.POINTER(C.c_uint8)]),
    "runner_forward_batch_logits": (_I, [_VP, _U32, _PU64, _PU32, _PU32, _PU32, C.POINTER(C.c_uint8),
                                         C.POINTER(C.c_float)]),
    "runner_forward_token": (_I, [_VP, _U64, _U32, _U32, _PU32, C.POINTER(C.c_float),
                                  C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), _PU32, _U32,
                                  C.POINTER(C.c_uint16)]),
    "runner_last_step_ms": (_F, [_VP]),
    "runner_last_launches": (_U32, [_VP]),
    "runner_last_transfer_bytes": (_I, [_VP, C.POINTER(_U64), C.POINTER(_U64)]),
    "runner_last_host_us": (_I, [_VP, C.POINTER(C.c_float)]),
    "runner_last_error": (_U32, [_VP, C.c_char_p, _U32]),
    "sched_create": (_VP, [_VP, _VP, _U32, _U32, _U64, _U32]),
    "sched_create_ex": (_VP, [_VP, _VP, _U32, _U32, _U64, _U32, _U32]),
    "sched_destroy": (None, [_VP]),
    "sched_submit_prefixed": (_I, [_VP, _U64, _PU32, _U32, _U32, _I64, _U32]),
    "sched_submit": (_I, [_VP, _U64, _PU32, _U32, _U32, _I64]),
    "sched_cancel": (_I, [_VP, _U64]),
    "sched_run_iteration": (None, [_VP, C.POINTER(Iteration)]),
    "sched_stop": (None, [_VP]),
    "sched_idle": (_I, [_VP]),
    "sched_drain": (_U32, [_VP, C.POINTER(Terminal), _U32, _PU32, _U32]),
    "sched_take_terminals": (_U32, [_VP, C.POINTER(Terminal), _U32, _PU32, _U32]),
    "generate": (_I, [_VP, _VP, _U64, _PU32, _U32, _U32, _I64, C.POINTER(Terminal), _PU32, _U32]),
    "fake_backend_create": (_VP, []),
    "fake_backend_destroy": (None, [_VP]),
    "fake_runner_create": (_VP, [_U32, _U32, _U32, _U32, _U64]),
    "fake_runner_destroy": (None, [_VP]),
    "fake_runner_log": (_U32, [_VP, _PU32, _U32, _PU64, _U32]),
}

_RUNTIME = None


def runtime() -> dict:
    """name -> ctypes function for every kkrt_* runtime entry point."""
    global _RUNTIME
    if _RUNTIME is None:
        _RUNTIME = bind(load_library(), "kkrt_", RUNTIME_SIGNATURES)
    return _RUNTIME


def _u32(seq):
    return (C.c_uint32 * max(len(seq), 1))(*seq)


def terminals_from(n, terms, tokens) -> list[dict]:
    out, at = [], 0
    for i in range(n):
        t = terms[i]
        out.append(dict(request_id=t.request_id, reason=t.reason, error=t.error,
                        tokens=list(tokens[at:at + t.token_count]), prompt_tokens=t.prompt_tokens,
                        completion_tokens=t.completion_tokens, ttft_ns=t.ttft_ns,
                        tpot_ns=t.tpot_ns, e2e_ns=t.e2e_ns))
        at += t.token_count
    return out


class Scheduler:
    """IterationSchedulerRuntime through the C ABI (kkrt_ = this library; the
    reference shim exposes the same calls with the kref_ prefix)."""

    def __init__(self, fns: dict, backend, runner, max_active, max_batched_tokens, max_kv_tokens,
                 prefill_chunk, fused_prefill=False):
        self.f = fns
        if fused_prefill:
            self.h = fns["sched_create_ex"](backend, runner, max_active, max_batched_tokens,
                                            max_kv_tokens, prefill_chunk, 1)
        else:
            self.h = fns["sched_create"](backend, runner, max_active, max_batched_tokens,
                                         max_kv_tokens, prefill_chunk)

    def submit(self, rid, prompt, max_new, eos=-1, kv_prefix=0):
        if kv_prefix:
            return self.f["sched_submit_prefixed"](self.h, rid, _u32(prompt), len(prompt), max_new, eos,
                                                   kv_prefix)
        return self.f["sched_submit"](self.h, rid, _u32(prompt), len(prompt), max_new, eos)

    def cancel(self, rid):
        return self.f["sched_cancel"](self.h, rid)

    def run_iteration(self):
        it = Iteration()
        self.f["sched_run_iteration"](self.h, C.byref(it))
        return _struct_tuple(it)

    def drain(self, cap=4096, token_cap=1 << 20):
        terms = (Terminal * cap)()
        toks = (C.c_uint32 * token_cap)()
        n = self.f["sched_drain"](self.h, terms, cap, toks, token_cap)
        return terminals_from(n, terms, toks)

    def stop(self):
        self.f["sched_stop"](self.h)

    def close(self):
        if self.h:
            self.f["sched_destroy"](self.h)
            self.h = None
