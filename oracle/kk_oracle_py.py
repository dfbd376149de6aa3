"""TEST INFRASTRUCTURE ONLY — ctypes bindings of the CPU oracle
(oracle/_build/libkk_oracle.so, a plain-C restatement of the reference
arithmetic; see kk_oracle.h) and of the reference shim
(oracle/_ref/libkimkv_ref.so, the reference's own sources). Imported only by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as checker."""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libkk_oracle.so"
REF_LIB = HERE / "_ref" / "libkimkv_ref.so"


def reference_dir() -> Path | None:
    """The reference source tree used to build oracle/_ref: the directory named
    by KK_REFERENCE_DIR, else BASELINE.json's `reference_path`; None when
    neither names an existing tree (as on a machine without the reference,
    where the prebuilt oracle/_ref library or the committed golden fixtures
    stand in)."""
    import json
    import os
    cand = os.environ.get("KK_REFERENCE_DIR")
    if not cand:
        baseline = HERE.parent / "BASELINE.json"
        if baseline.exists():
            cand = json.loads(baseline.read_text()).get("reference_path")
    if cand and (Path(cand) / "src").is_dir():
        return Path(cand)
    return None


def build_ref() -> bool:
    """Builds oracle/_ref from the reference tree when one is available."""
    ref = reference_dir()
    if ref is None:
        return False
    subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True,
                   capture_output=True)
    return REF_LIB.exists()


class Config(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("layers", C.c_uint32),
                ("q_heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("vocab", C.c_uint32), ("max_positions", C.c_uint32), ("eps", C.c_float),
                ("theta", C.c_float)]


_lib = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = C.CDLL(str(LIB))
        u16p, f32p, u32p, u64p = (C.POINTER(C.c_uint16), C.POINTER(C.c_float),
                                  C.POINTER(C.c_uint32), C.POINTER(C.c_uint64))
        sig = {
            "kko_f2h": (C.c_uint16, [C.c_float]),
            "kko_h2f": (C.c_float, [C.c_uint16]),
            "kko_reference_attention": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, u16p,
                                                  C.c_uint32, f32p, f32p]),
            "kko_paged_attention": (C.c_int, [u16p, u16p, C.c_uint32, C.c_uint32, C.c_uint32,
                                              C.c_uint32, C.c_uint32, u32p, u32p,
                                              C.POINTER(C.c_uint8), C.c_uint32, u16p, u16p]),
            "kko_model_create": (C.c_void_p, [C.POINTER(Config), C.POINTER(u16p), C.c_uint32]),
            "kko_model_destroy": (None, [C.c_void_p]),
            "kko_seq_create": (C.c_int, [C.c_void_p, C.c_uint64]),
            "kko_seq_fork": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64]),
            "kko_seq_release": (C.c_int, [C.c_void_p, C.c_uint64]),
            "kko_seq_length": (C.c_uint32, [C.c_void_p, C.c_uint64]),
            "kko_seq_append_kv": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint32, u16p, u16p]),
            "kko_forward_batch": (C.c_int, [C.c_void_p, C.c_uint32, u64p, u32p, u32p, f32p, u16p,
                                            u32p]),
            "kko_argmax": (C.c_uint32, [f32p, C.c_uint32]),
            "kko_model_set_wide_sums": (None, [C.c_void_p, C.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        _lib = lib
    return _lib


def ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


def reference_attention(kv: np.ndarray, tokens: int, query: np.ndarray, layers: int, heads: int,
                        dim: int, lib=None) -> np.ndarray | None:
    lib = lib or load()
    out = np.zeros(layers * heads * dim, dtype=np.float32)
    kv = np.ascontiguousarray(kv, dtype=np.uint16)
    query = np.ascontiguousarray(query, dtype=np.float32)
    ok = lib.kko_reference_attention(layers, heads, dim, ptr(kv, C.c_uint16), tokens,
                                     ptr(query, C.c_float), ptr(out, C.c_float))
    return out if ok else None


def paged_attention(micro: np.ndarray, extent: np.ndarray, layers, kv_heads, dim, layer, q_heads,
                    table, q: np.ndarray) -> np.ndarray:
    """table: list of (slot, begin, valid, kind); q: [q_heads*dim] uint16."""
    lib = load()
    slot = np.array([e[0] for e in table], dtype=np.uint32)
    valid = np.array([e[2] for e in table], dtype=np.uint32)
    kind = np.array([e[3] for e in table], dtype=np.uint8)
    out = np.zeros(q_heads * dim, dtype=np.uint16)
    micro = np.ascontiguousarray(micro, dtype=np.uint16)
    extent = np.ascontiguousarray(extent, dtype=np.uint16)
    q = np.ascontiguousarray(q, dtype=np.uint16)
    ok = lib.kko_paged_attention(ptr(micro, C.c_uint16), ptr(extent, C.c_uint16), layers, kv_heads,
                                 dim, layer, q_heads, ptr(slot, C.c_uint32), ptr(valid, C.c_uint32),
                                 ptr(kind, C.c_uint8), len(table), ptr(q, C.c_uint16),
                                 ptr(out, C.c_uint16))
    assert ok
    return out


class Model:
    """The FP16-rounding decoder oracle over numpy FP16 (uint16) weights in the
    order documented in kk_oracle.h."""

    def __init__(self, cfg: dict, weights: list, threads: int = 8):
        self.lib = load()
        self.cfg = cfg
        c = Config(cfg["hidden"], cfg["intermediate"], cfg["layers"], cfg["q_heads"],
                   cfg["kv_heads"], cfg["head_dim"], cfg["vocab"], cfg["max_positions"],
                   cfg["eps"], cfg["theta"])
        self._keep = [np.ascontiguousarray(w, dtype=np.uint16) for w in weights]
        arr = (C.POINTER(C.c_uint16) * len(self._keep))(*[ptr(w, C.c_uint16) for w in self._keep])
        self.h = self.lib.kko_model_create(C.byref(c), arr, threads)
        self._keep = None  # widened copies live in the oracle now
        assert self.h

    def close(self):
        if self.h:
            self.lib.kko_model_destroy(self.h)
            self.h = None

    __del__ = close

    def create(self, seq):
        assert self.lib.kko_seq_create(self.h, seq)

    def fork(self, src, child):
        assert self.lib.kko_seq_fork(self.h, src, child)

    def release(self, seq):
        self.lib.kko_seq_release(self.h, seq)

    def length(self, seq):
        return self.lib.kko_seq_length(self.h, seq)

    def append_kv(self, seq, k: np.ndarray, v: np.ndarray):
        k = np.ascontiguousarray(k, dtype=np.uint16)
        v = np.ascontiguousarray(v, dtype=np.uint16)
        n = k.shape[0]
        assert self.lib.kko_seq_append_kv(self.h, seq, n, ptr(k, C.c_uint16), ptr(v, C.c_uint16))

    def set_wide_sums(self, wide: bool):
        self.lib.kko_model_set_wide_sums(self.h, 1 if wide else 0)

    def forward(self, seqs, tokens, positions, want_logits=True, want_hidden=True):
        n = len(seqs)
        ids = np.array(seqs, dtype=np.uint64)
        tok = np.array(tokens, dtype=np.uint32)
        pos = np.array(positions, dtype=np.uint32)
        logits = np.zeros((n, self.cfg["vocab"]), dtype=np.float32) if want_logits else None
        hidden = np.zeros((n, self.cfg["hidden"]), dtype=np.uint16) if want_hidden else None
        greedy = np.zeros(n, dtype=np.uint32)
        ok = self.lib.kko_forward_batch(
            self.h, n, ptr(ids, C.c_uint64), ptr(tok, C.c_uint32), ptr(pos, C.c_uint32),
            ptr(logits, C.c_float) if logits is not None else None,
            ptr(hidden, C.c_uint16) if hidden is not None else None, ptr(greedy, C.c_uint32))
        assert ok, "oracle forward rejected its inputs"
        return greedy, logits, hidden


class RefModelConfig(C.Structure):
    _fields_ = Config._fields_


class RefModel:
    """The reference's own model oracle (ReferenceModel of the reference's
    runner contract test, compiled into oracle/_ref by ref_model_shim.cpp):
    the contract archive with the reference test's weights (cfg None), or a
    config whose weights are the given FP16 tensors (oracle order)."""

    def __init__(self, cfg: dict | None = None, weights: list | None = None):
        import tempfile
        lib = C.CDLL(str(REF_LIB))
        u16p = C.POINTER(C.c_uint16)
        sig = {
            "kref_model_create": (C.c_void_p, [C.POINTER(RefModelConfig), C.POINTER(u16p), C.c_char_p]),
            "kref_model_destroy": (None, [C.c_void_p]),
            "kref_model_config_of": (None, [C.c_void_p, C.POINTER(RefModelConfig)]),
            "kref_model_tensor_count": (C.c_uint32, [C.c_void_p]),
            "kref_model_tensor": (C.c_uint64, [C.c_void_p, C.c_uint32, u16p]),
            "kref_model_forward": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_float),
                                             u16p]),
            "kref_model_generate": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.c_uint32, C.c_uint32,
                                              C.POINTER(C.c_uint32)]),
            "kref_model_lane_create": (C.c_void_p, [C.c_void_p]),
            "kref_model_lane_destroy": (None, [C.c_void_p]),
            "kref_model_lane_length": (C.c_uint32, [C.c_void_p]),
            "kref_model_lane_append_kv": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, u16p, u16p]),
            "kref_model_forward_lanes": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p),
                                                   C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                                   C.POINTER(C.c_uint32), C.c_uint32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        self.lib = lib
        self.lanes = []
        scratch = tempfile.gettempdir().encode()
        if cfg is None:
            self.h = lib.kref_model_create(None, None, scratch)
        else:
            c = RefModelConfig(cfg["hidden"], cfg["intermediate"], cfg["layers"], cfg["q_heads"],
                               cfg["kv_heads"], cfg["head_dim"], cfg["vocab"], cfg["max_positions"],
                               cfg["eps"], cfg["theta"])
            keep = [np.ascontiguousarray(w, dtype=np.uint16).ravel() for w in weights]
            arr = (u16p * len(keep))(*[ptr(w, C.c_uint16) for w in keep])
            self.h = lib.kref_model_create(C.byref(c), arr, scratch)
        assert self.h
        out = RefModelConfig()
        lib.kref_model_config_of(self.h, C.byref(out))
        self.cfg = {name: getattr(out, name) for name, _ in RefModelConfig._fields_}

    def tensors(self) -> list:
        out = []
        for i in range(self.lib.kref_model_tensor_count(self.h)):
            n = self.lib.kref_model_tensor(self.h, i, None)
            t = np.zeros(n, dtype=np.uint16)
            self.lib.kref_model_tensor(self.h, i, ptr(t, C.c_uint16))
            out.append(t)
        return out

    def forward(self, token: int, position: int):
        logits = np.zeros(self.cfg["vocab"], dtype=np.float32)
        hidden = np.zeros(self.cfg["hidden"], dtype=np.uint16)
        assert self.lib.kref_model_forward(self.h, token, position, ptr(logits, C.c_float),
                                           ptr(hidden, C.c_uint16))
        return logits, hidden

    def generate(self, prompt: list, max_new: int) -> list:
        out = (C.c_uint32 * max_new)()
        n = self.lib.kref_model_generate(self.h, (C.c_uint32 * len(prompt))(*prompt), len(prompt),
                                         max_new, out)
        return [out[i] for i in range(n)]

    # Lanes: more ReferenceModel instances over this archive (own K/V each).
    def lane_create(self) -> int:
        lane = self.lib.kref_model_lane_create(self.h)
        assert lane
        self.lanes.append(lane)
        return lane

    def lane_append_kv(self, lane: int, k: np.ndarray, v: np.ndarray):
        """k, v: FP16 bits [n][layers][kv_heads * head_dim]."""
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        assert self.lib.kref_model_lane_append_kv(self.h, lane, k.shape[0], ptr(k, C.c_uint16),
                                                  ptr(v, C.c_uint16))

    def lane_length(self, lane: int) -> int:
        return self.lib.kref_model_lane_length(lane)

    def forward_lanes(self, lanes: list, tokens: list, positions: list, threads: int) -> list:
        """ReferenceModel::forward once per lane, over `threads` host threads;
        the greedy token of each lane."""
        n = len(lanes)
        out = (C.c_uint32 * n)()
        assert self.lib.kref_model_forward_lanes(self.h, n, (C.c_void_p * n)(*lanes),
                                                 (C.c_uint32 * n)(*tokens), (C.c_uint32 * n)(*positions),
                                                 out, threads), "reference forward rejected its inputs"
        return list(out)

    def close(self):
        for lane in getattr(self, "lanes", []):
            self.lib.kref_model_lane_destroy(lane)
        self.lanes = []
        if getattr(self, "h", None):
            self.lib.kref_model_destroy(self.h)
            self.h = None

    __del__ = close
