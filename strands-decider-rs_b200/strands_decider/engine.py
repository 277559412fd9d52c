"""ctypes binding of the C ABI in include/sd_b200.h (libsdb200.so, built from ../csrc).

`Engine` mirrors the reference's `Engine` (`src/engine.rs:175,305,529`): `load`, `hidden_size`,
`forward(ids, rows, cache, keep, timed)` returning an `Output`, and immutable `Snapshot`s. `Head`
mirrors `src/head.rs`. There is no fallback: without the native library every call raises.
"""
from __future__ import annotations

import ctypes as C
import json
import os
from dataclasses import dataclass

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG, "libsdb200.so")

SD_OK = 0
CONTEXT = 4096  # `src/engine.rs:16`


class Error(RuntimeError):
    """The reference's `Error(String)` (`src/lib.rs:23-44`), with the C ABI's status code."""

    def __init__(self, msg: str, code: int = -1):
        super().__init__(msg)
        self.code = code


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise Error(f"{LIB_PATH} is missing: build it with `make -C {os.path.join(PKG, 'csrc')}` "
                        "(or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        vp, i32, cp = C.c_void_p, C.c_int32, C.c_char_p
        L.sd_last_error.restype = cp
        L.sd_engine_create.argtypes = [cp, C.c_int, C.POINTER(vp)]
        L.sd_engine_destroy.argtypes = [vp]
        L.sd_engine_hidden_size.argtypes = [vp]
        L.sd_engine_num_layers.argtypes = [vp]
        L.sd_engine_last_error.restype = cp
        L.sd_engine_last_error.argtypes = [vp]
        L.sd_engine_set_trace.argtypes = [vp, vp, C.c_size_t]
        L.sd_forward.argtypes = [vp, vp, i32, vp, i32, vp, i32, vp, C.POINTER(vp), C.POINTER(C.c_double)]
        L.sd_forward_dev.argtypes = [vp, vp, i32, vp, i32, vp, i32, vp, C.POINTER(vp)]
        L.sd_forward_fork.argtypes = [vp, vp, vp, vp, i32, vp, vp, vp, C.POINTER(C.c_double)]
        L.sd_forward_fork_dev.argtypes = [vp, vp, vp, vp, i32, vp, vp, vp]
        L.sd_forward_fork_multi.argtypes = [vp, vp, vp, vp, i32, vp, vp, vp, C.POINTER(C.c_double)]
        L.sd_forward_fork_multi_dev.argtypes = [vp, vp, vp, vp, i32, vp, vp, vp]
        L.sd_forward_batch.argtypes = [vp, vp, vp, vp, i32, vp, vp, i32, vp, vp, C.POINTER(C.c_double)]
        L.sd_engine_reserve.argtypes = [vp, i32, i32, i32]
        L.sd_forward_batch_dev.argtypes = [vp, vp, vp, vp, i32, vp, vp, i32, vp, vp]
        L.sd_engine_synchronize.argtypes = [vp]
        L.sd_engine_stream.restype = vp
        L.sd_engine_stream.argtypes = [vp]
        L.sd_engine_launches.restype = C.c_int64
        L.sd_engine_launches.argtypes = [vp]
        L.sd_engine_profile.argtypes = [vp, i32]
        L.sd_engine_profile_get.argtypes = [vp, i32, C.POINTER(C.c_double), C.POINTER(C.c_int64), C.POINTER(C.c_double)]
        L.sd_snapshot_len.restype = i32
        L.sd_snapshot_len.argtypes = [vp]
        L.sd_snapshot_free.argtypes = [vp]
        L.sd_head_load.argtypes = [cp, C.POINTER(vp)]
        L.sd_head_free.argtypes = [vp]
        L.sd_head_probs.argtypes = [vp, vp, i32, i32, C.c_double, vp]
        L.sd_head_probs_dev.argtypes = [vp, vp, vp, vp, i32, vp, vp]
        L.sd_decode_scales.argtypes = [vp, i32, i32, vp, vp]
        L.sd_forward_fork_multi_probs.argtypes = [vp, vp, vp, vp, i32, vp, vp, vp, vp, vp]
        L.sd_forward_tree.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp, vp]
        L.sd_forward_tree_probs.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp, vp, vp, vp]
        L.sd_forward_tree_dev.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp, vp]
        L.sd_attention.argtypes = [vp, vp, vp, vp, i32, i32, i32, vp, i32, i32, i32, i32, i32, i32, vp]
        L.sd_attention_batch.argtypes = [vp, vp, vp, vp, i32, i32, i32, vp, i32, i32, i32, i32, i32, i32, i32, vp]
        L.sd_attention_split.argtypes = [vp, vp, vp, vp, i32, i32, i32, vp, i32, i32, i32, i32, i32, i32, i32, vp,
                                         C.c_size_t, vp]
        L.sd_gdn.argtypes = [vp, vp, i32, vp, i32, vp, vp, vp, i32, vp, i32, i32, i32, C.c_int64, C.c_int64, i32, i32, vp,
                             C.c_size_t, vp]
        L.sd_gdn_noalloc.argtypes = [vp, vp, i32, vp, i32, vp, vp, vp, i32, vp, i32, i32, vp]
        L.sd_gdn_noalloc_max_tokens.restype = i32
        L.sd_gdn_noalloc_max_tokens.argtypes = [i32]
        L.sd_gdn_scratch_bytes.restype = C.c_size_t
        L.sd_gdn_scratch_bytes.argtypes = [i32, i32]
        L.sd_qweight_create.argtypes = [vp, vp, i32, i32, i32, C.POINTER(vp)]
        L.sd_engine_selftest_wait.argtypes = [vp, i32]
        L.sd_op_status.argtypes = [vp]
        L.sd_qweight_create_format.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, C.POINTER(vp)]
        L.sd_qweight_free.argtypes = [vp]
        L.sd_matmul.argtypes = [vp, vp, i32, vp, i32, i32, vp, C.c_size_t, vp]
        L.sd_matmul_ex.argtypes = [vp, vp, i32, vp, i32, i32, vp, vp, C.c_size_t, i32, vp]
        L.sd_decider_load.argtypes = [cp, C.c_int, C.POINTER(vp)]
        L.sd_decider_free.argtypes = [vp]
        L.sd_decider_ask_all.argtypes = [vp, cp, C.POINTER(vp)]
        L.sd_decider_ask_batch.argtypes = [vp, cp, C.POINTER(vp)]
        L.sd_decider_last_error.argtypes = [vp]
        L.sd_decider_last_error.restype = cp
        L.sd_host_last_error.restype = cp
        L.sd_string_free.argtypes = [vp]
        _lib = L
    return _lib


def _check(rc: int, what: str, engine=None):
    if rc != SD_OK:
        L = lib()
        msg = (L.sd_engine_last_error(engine) if engine else L.sd_last_error()).decode(errors="replace")
        raise Error(f"{what}: {msg}", rc)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


class Snapshot:
    """The torso state after a prefix (`src/engine.rs:80-87`): immutable, reusable, freed with it."""

    def __init__(self, handle: int):
        self._h = handle

    @property
    def len(self) -> int:
        return lib().sd_snapshot_len(self._h)

    def close(self):
        if self._h:
            lib().sd_snapshot_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class Output:
    """`Output` (`src/engine.rs:88-96`): hidden rows [rows, d] f32, GPU time, optional snapshot."""
    hidden: np.ndarray
    d: int
    gpu_ms: float | None
    snapshot: Snapshot | None


class Engine:
    """The torso on one B200 (`Engine`, `src/engine.rs`)."""

    def __init__(self, handle: int, device: int):
        self._h = handle
        self.device = device
        self.adapter = f"NVIDIA B200 (cuda:{device}, sm_100a)"
        self._trace = None

    @classmethod
    def load(cls, model_dir: str, device: int = 0) -> "Engine":
        """`Engine::load` (`src/engine.rs:175-303`)."""
        h = C.c_void_p()
        _check(lib().sd_engine_create(os.fsencode(model_dir), device, C.byref(h)), "Engine::load")
        return cls(h.value, device)

    def hidden_size(self) -> int:
        return lib().sd_engine_hidden_size(self._h)

    def num_layers(self) -> int:
        return lib().sd_engine_num_layers(self._h)

    def forward(self, ids, rows, cache: Snapshot | None = None, keep: bool = False, timed: bool = False,
                trace: bool = False) -> Output:
        """`Engine::forward` (`src/engine.rs:529-662`). With ``trace``, ``Output.trace`` holds the
        residual stream after each layer [n_layers, n_ids, d]."""
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = np.ascontiguousarray(rows, np.int32)
        d = self.hidden_size()
        hidden = np.zeros((len(rows), d), np.float32)
        snap = C.c_void_p()
        ms = C.c_double(0.0)
        L = lib()
        tr = None
        if trace:
            tr = np.zeros((self.num_layers(), len(ids), d), np.float32)
            _check(L.sd_engine_set_trace(self._h, _ptr(tr), tr.size), "trace", self._h)
        try:
            rc = L.sd_forward(self._h, _ptr(ids), len(ids), _ptr(rows) if len(rows) else None, len(rows),
                              cache._h if cache is not None else None, int(keep), _ptr(hidden) if len(rows) else None,
                              C.byref(snap), C.byref(ms))
        finally:
            if trace:
                L.sd_engine_set_trace(self._h, None, 0)
        _check(rc, "Engine::forward", self._h)
        out = Output(hidden, d, ms.value if timed else None, Snapshot(snap.value) if keep else None)
        out.trace = tr
        return out

    def forward_fork(self, cache, ids_list, rows_list, timed: bool = False):
        """`sd_forward_fork`: every question (ids_list[b], its rows rows_list[b]) continued from the
        snapshot ``cache`` in one pass; ``cache`` a list of snapshots, one per question
        (`sd_forward_fork_multi`): questions of several requests in one pass. Returns the hidden
        rows of each question ([rows, d] f32 each) and, with ``timed``, the pass's device time in ms."""
        lens = np.array([len(x) for x in ids_list], np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(x, np.uint32) for x in ids_list]), np.uint32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list] + [np.zeros(0, np.int32)]),
                                    np.int32)
        d = self.hidden_size()
        hidden = np.zeros((int(nrows.sum()), d), np.float32)
        ms = C.c_double(0.0)
        if isinstance(cache, (list, tuple)):
            caches = (C.c_void_p * len(cache))(*[c._h for c in cache])
            _check(lib().sd_forward_fork_multi(self._h, caches, _ptr(ids), _ptr(lens), len(lens),
                                               _ptr(rows) if len(rows) else None, _ptr(nrows),
                                               _ptr(hidden) if len(rows) else None, C.byref(ms)),
                   "sd_forward_fork_multi", self._h)
        else:
            _check(lib().sd_forward_fork(self._h, cache._h, _ptr(ids), _ptr(lens), len(lens), _ptr(rows) if len(rows) else None,
                                         _ptr(nrows), _ptr(hidden) if len(rows) else None, C.byref(ms)),
                   "sd_forward_fork", self._h)
        outs = np.split(hidden, np.cumsum(nrows)[:-1]) if len(nrows) > 1 else [hidden]
        return (outs, ms.value) if timed else outs

    def forward_fork_dev(self, cache, ids_dev: int, lens, rows_list, hidden_dev: int | None):
        """`sd_forward_fork_dev`: the fork with the questions' ids on the GPU (back to back, lens[b]
        each), hidden rows to ``hidden_dev``, queued on the engine's stream; ``cache`` a snapshot or
        one per question (`sd_forward_fork_multi_dev`)."""
        lens = np.ascontiguousarray(lens, np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list] + [np.zeros(0, np.int32)]),
                                    np.int32)
        if isinstance(cache, (list, tuple)):
            caches = (C.c_void_p * len(cache))(*[c._h for c in cache])
            _check(lib().sd_forward_fork_multi_dev(self._h, caches, ids_dev, _ptr(lens), len(lens),
                                                   _ptr(rows) if len(rows) else None, _ptr(nrows), hidden_dev),
                   "sd_forward_fork_multi_dev", self._h)
        else:
            _check(lib().sd_forward_fork_dev(self._h, cache._h, ids_dev, _ptr(lens), len(lens),
                                             _ptr(rows) if len(rows) else None, _ptr(nrows), hidden_dev),
                   "sd_forward_fork_dev", self._h)

    def forward_fork_probs(self, caches, ids_list, rows_list, head: "Head", temperatures):
        """`sd_forward_fork_multi_probs`: question b (ids_list[b], its option rows then its answer
        row in rows_list[b]) continued from caches[b], then the pointer head on the GPU; returns each
        question's probabilities (f64, len(rows_list[b]) - 1 each)."""
        lens = np.array([len(x) for x in ids_list], np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(x, np.uint32) for x in ids_list]), np.uint32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list]), np.int32)
        temps = np.ascontiguousarray(np.broadcast_to(np.asarray(temperatures, np.float64), (len(lens),)))
        probs = np.zeros(int(nrows.sum()) - len(lens), np.float64)
        caches = (C.c_void_p * len(caches))(*[c._h for c in caches])
        _check(lib().sd_forward_fork_multi_probs(self._h, caches, _ptr(ids), _ptr(lens), len(lens), _ptr(rows), _ptr(nrows),
                                                 head._h, _ptr(temps), _ptr(probs)),
               "sd_forward_fork_multi_probs", self._h)
        return np.split(probs, np.cumsum(nrows - 1)[:-1]) if len(lens) > 1 else [probs]

    def _tree_args(self, caches, parents, ids_list, rows_list):
        n = len(ids_list)
        lens = np.array([len(x) for x in ids_list], np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        par = np.ascontiguousarray(parents, np.int32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(x, np.uint32) for x in ids_list]), np.uint32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list] + [np.zeros(0, np.int32)]),
                                    np.int32)
        cs = None if caches is None else (C.c_void_p * n)(*[c._h if c is not None else None for c in caches])
        return n, lens, nrows, par, ids, rows, cs

    def forward_tree(self, caches, parents, ids_list, rows_list):
        """`sd_forward_tree`: one packed pass in which sequence b continues caches[b] (None: fresh) or,
        with parents[b] >= 0, the earlier sequence parents[b] of the same pass (a request's questions
        after its state). Returns the hidden rows of each sequence."""
        n, lens, nrows, par, ids, rows, cs = self._tree_args(caches, parents, ids_list, rows_list)
        hidden = np.zeros((int(nrows.sum()), self.hidden_size()), np.float32)
        _check(lib().sd_forward_tree(self._h, cs, _ptr(par), _ptr(ids), _ptr(lens), n, _ptr(rows) if len(rows) else None,
                                     _ptr(nrows), _ptr(hidden) if len(rows) else None),
               "sd_forward_tree", self._h)
        return np.split(hidden, np.cumsum(nrows)[:-1]) if n > 1 else [hidden]

    def forward_tree_dev(self, caches, parents, ids_dev: int, lens, rows_list, hidden_dev: int | None):
        """`sd_forward_tree_dev`: forward_tree with the ids already on the GPU (int32, back to back) and
        the rows written to ``hidden_dev``, queued on the engine's stream."""
        n = len(lens)
        lens = np.ascontiguousarray(lens, np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        par = np.ascontiguousarray(parents, np.int32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list] + [np.zeros(0, np.int32)]),
                                    np.int32)
        cs = None if caches is None else (C.c_void_p * n)(*[c._h if c is not None else None for c in caches])
        _check(lib().sd_forward_tree_dev(self._h, cs, _ptr(par), ids_dev, _ptr(lens), n, _ptr(rows) if len(rows) else None,
                                         _ptr(nrows), hidden_dev),
               "sd_forward_tree_dev", self._h)

    def forward_tree_probs(self, caches, parents, ids_list, rows_list, head: "Head", temperatures):
        """`sd_forward_tree_probs`: the tree pass of forward_tree, then the pointer head on the GPU over
        the sequences with rows (options then the answer row); returns their probabilities in order."""
        n, lens, nrows, par, ids, rows, cs = self._tree_args(caches, parents, ids_list, rows_list)
        temps = np.ascontiguousarray(np.broadcast_to(np.asarray(temperatures, np.float64), (n,)))
        asked = nrows[nrows > 0]
        probs = np.zeros(int(asked.sum()) - len(asked), np.float64)
        _check(lib().sd_forward_tree_probs(self._h, cs, _ptr(par), _ptr(ids), _ptr(lens), n, _ptr(rows), _ptr(nrows),
                                           head._h, _ptr(temps), _ptr(probs)),
               "sd_forward_tree_probs", self._h)
        return np.split(probs, np.cumsum(asked - 1)[:-1]) if len(asked) > 1 else [probs]

    def head_probs_dev(self, head: "Head", hidden_dev: int, nrows, temperatures, probs_dev: int):
        """`sd_head_probs_dev`: the pointer head over questions' rows already on the GPU (question b:
        nrows[b] rows at ``hidden_dev``, back to back), probabilities to ``probs_dev`` (f64), queued on
        the engine's stream."""
        nrows = np.ascontiguousarray(nrows, np.int32)
        temps = np.ascontiguousarray(np.broadcast_to(np.asarray(temperatures, np.float64), (len(nrows),)))
        _check(lib().sd_head_probs_dev(self._h, head._h, hidden_dev, _ptr(nrows), len(nrows), _ptr(temps), probs_dev),
               "sd_head_probs_dev", self._h)

    def reserve(self, max_tokens: int, max_seqs: int, max_rows: int):
        """`sd_engine_reserve`: size the working memory for passes up to these bounds up front."""
        _check(lib().sd_engine_reserve(self._h, max_tokens, max_seqs, max_rows), "sd_engine_reserve", self._h)

    def forward_batch(self, caches, ids_list, rows_list, keep: bool = False, timed: bool = False):
        """`sd_forward_batch`: sequence b (ids_list[b], rows rows_list[b]) continuing caches[b] (None:
        a fresh sequence; ``caches`` None: all fresh), all in one pass. Returns the hidden rows of
        each sequence, the new snapshots (with ``keep``; else None) and, with ``timed``, the device
        time in ms."""
        n = len(ids_list)
        lens = np.array([len(x) for x in ids_list], np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(x, np.uint32) for x in ids_list]), np.uint32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list] + [np.zeros(0, np.int32)]),
                                    np.int32)
        hidden = np.zeros((int(nrows.sum()), self.hidden_size()), np.float32)
        cs = None if caches is None else (C.c_void_p * n)(*[c._h if c is not None else None for c in caches])
        out = (C.c_void_p * n)()
        ms = C.c_double(0.0)
        _check(lib().sd_forward_batch(self._h, cs, _ptr(ids), _ptr(lens), n, _ptr(rows) if len(rows) else None, _ptr(nrows),
                                      int(keep), _ptr(hidden) if len(rows) else None, out if keep else None, C.byref(ms)),
               "sd_forward_batch", self._h)
        outs = np.split(hidden, np.cumsum(nrows)[:-1]) if n > 1 else [hidden]
        snaps = [Snapshot(out[b]) for b in range(n)] if keep else None
        return (outs, snaps, ms.value) if timed else (outs, snaps)

    def forward_batch_dev(self, caches, ids_dev: int, lens, rows_list, hidden_dev: int | None, keep: bool = False):
        """`sd_forward_batch_dev`: the batch with the ids on the GPU (back to back), rows to
        ``hidden_dev``, queued on the engine's stream. Returns the new snapshots (with ``keep``)."""
        n = len(lens)
        lens = np.ascontiguousarray(lens, np.int32)
        nrows = np.array([len(r) for r in rows_list], np.int32)
        rows = np.ascontiguousarray(np.concatenate([np.asarray(r, np.int32) for r in rows_list] + [np.zeros(0, np.int32)]),
                                    np.int32)
        cs = None if caches is None else (C.c_void_p * n)(*[c._h if c is not None else None for c in caches])
        out = (C.c_void_p * n)()
        _check(lib().sd_forward_batch_dev(self._h, cs, ids_dev, _ptr(lens), n, _ptr(rows) if len(rows) else None, _ptr(nrows),
                                          int(keep), hidden_dev, out if keep else None), "sd_forward_batch_dev", self._h)
        return [Snapshot(out[b]) for b in range(n)] if keep else None

    def forward_dev(self, ids_dev: int, n_ids: int, rows_dev: int | None, n_rows: int, cache: Snapshot | None = None,
                    keep: bool = False, hidden_dev: int | None = None) -> Snapshot | None:
        """`sd_forward_dev`: the forward on device buffers, queued on the engine's stream."""
        snap = C.c_void_p()
        _check(lib().sd_forward_dev(self._h, ids_dev, n_ids, rows_dev, n_rows, cache._h if cache is not None else None,
                                    int(keep), hidden_dev, C.byref(snap)), "sd_forward_dev", self._h)
        return Snapshot(snap.value) if keep else None

    def selftest_wait(self, limit_us: int):
        """`sd_engine_selftest_wait`: a bounded wait that runs out on purpose; raises the kernel error."""
        _check(lib().sd_engine_selftest_wait(self._h, limit_us), "selftest", self._h)

    def synchronize(self):
        _check(lib().sd_engine_synchronize(self._h), "sd_engine_synchronize", self._h)

    @property
    def stream(self) -> int:
        return lib().sd_engine_stream(self._h) or 0

    def launches(self) -> int:
        return int(lib().sd_engine_launches(self._h))

    PROFILE_KINDS = ("gemm", "attention", "gdn", "other")

    def profile(self, enable: bool):
        """Per-kernel-kind device time (the reference's `Engine::profile`, `src/engine.rs:665-711`)."""
        _check(lib().sd_engine_profile(self._h, int(enable)), "sd_engine_profile", self._h)

    def profile_get(self) -> dict:
        out = {}
        for i, name in enumerate(self.PROFILE_KINDS):
            ms, n, work = C.c_double(), C.c_int64(), C.c_double()
            _check(lib().sd_engine_profile_get(self._h, i, C.byref(ms), C.byref(n), C.byref(work)), "profile", self._h)
            out[name] = {"ms": ms.value, "launches": n.value, "work": work.value}
        return out

    def close(self):
        if self._h:
            lib().sd_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Head:
    """The pointer head (`src/head.rs`), in f64 on the host."""

    def __init__(self, handle: int):
        self._h = handle

    @classmethod
    def load(cls, path: str) -> "Head":
        h = C.c_void_p()
        _check(lib().sd_head_load(os.fsencode(path), C.byref(h)), "Head::load")
        return cls(h.value)

    def probs(self, hidden: np.ndarray, d: int, temperature: float) -> np.ndarray:
        hidden = np.ascontiguousarray(hidden, np.float32).reshape(-1, d)
        out = np.zeros(hidden.shape[0] - 1, np.float64)
        _check(lib().sd_head_probs(self._h, _ptr(hidden), hidden.shape[0], d, float(temperature), _ptr(out)), "Head::probs")
        return out

    def __del__(self):
        try:
            if self._h:
                lib().sd_head_free(self._h)
        except Exception:
            pass


# ---------------------------------------------------------------------------------------------
# Kernel-level entry points on device memory (pointers as ints, e.g. torch.Tensor.data_ptr())
# ---------------------------------------------------------------------------------------------

def attention_batch(q, k, v, gate, gstride, goff, gstep, out, batch, l, p, lt, hq, hk, hd, stream=None):
    """`sd_attention_batch`: `batch` sequences in one launch (q [batch][hq][l][hd], k/v [batch][hk][lt][hd])."""
    _check(lib().sd_attention_batch(q, k, v, gate, gstride, goff, gstep, out, batch, l, p, lt, hq, hk, hd, stream),
           "sd_attention_batch")


def attention(q, k, v, gate, gstride, goff, gstep, out, l, p, lt, hq, hk, hd, stream=None, splits=None, ws=None,
              ws_bytes=0):
    """`sd_attention`; with ``splits`` (0: the engine's choice), `sd_attention_split` on workspace ``ws``."""
    if splits is None:
        _check(lib().sd_attention(q, k, v, gate, gstride, goff, gstep, out, l, p, lt, hq, hk, hd, stream), "sd_attention")
    else:
        _check(lib().sd_attention_split(q, k, v, gate, gstride, goff, gstep, out, l, p, lt, hq, hk, hd, splits, ws,
                                        ws_bytes, stream), "sd_attention_split")


GDN_CHUNKED, GDN_SERIAL, GDN_TWO_PHASE = 0, 1, 2


def gdn(q, k, qk_stride, v, v_stride, beta, g, state, load_state, o, l, h, batch=1, seq_qk=0, seq_v=0, in_f16=False,
        serial=False, algo=None, scratch=None, scratch_bytes=0, stream=None):
    """`sd_gdn`: g is the log decay (decay = exp(g)); algo 0 chunked, 1 token-serial, 2 two-phase."""
    if algo is None:
        algo = GDN_SERIAL if serial else GDN_CHUNKED
    _check(lib().sd_gdn(q, k, qk_stride, v, v_stride, beta, g, state, int(load_state), o, l, h, batch, seq_qk, seq_v,
                        int(in_f16), int(algo), scratch, scratch_bytes, stream), "sd_gdn")


def op_status(stream=None):
    """`sd_op_status`: synchronises ``stream`` and raises if a kernel of a standalone call (gdn,
    attention, matmul) gave up on a bounded wait since the last check."""
    _check(lib().sd_op_status(stream), "sd_op_status")


def decode_scales(src, n, g, dst, stream=None):
    """`decode_scales` (`src/model.rs:219-236`) on the device: n headers then n x g codes at ``src``,
    [n][g] fp16 to ``dst`` (device pointers)."""
    _check(lib().sd_decode_scales(src, n, g, dst, stream), "sd_decode_scales")


def gdn_scratch_bytes(l: int, h: int) -> int:
    return int(lib().sd_gdn_scratch_bytes(l, h))


def gdn_noalloc(q, k, qk_stride, v, v_stride, beta, g, state, load_state, o, l, h, stream=None):
    """`sd_gdn_noalloc`: the two-phase scan on the library's fixed scratch array (no allocation)."""
    _check(lib().sd_gdn_noalloc(q, k, qk_stride, v, v_stride, beta, g, state, int(load_state), o, l, h, stream),
           "sd_gdn_noalloc")


def gdn_noalloc_max_tokens(h: int) -> int:
    return int(lib().sd_gdn_noalloc_max_tokens(h))


class QWeight:
    def __init__(self, q_dev: int, s_dev: int, n: int, k: int, interleave: bool = False, bits: int = 4, group: int = 32,
                 b_dev: int | None = None):
        """A weight in the reference's block-quantized layout (int2/int3/int4, one f16 scale per `group`
        weights, and with ``b_dev`` one f16 bias per group: asymmetric), repacked for the GEMM
        (`sd_qweight_create_format`)."""
        h = C.c_void_p()
        _check(lib().sd_qweight_create_format(q_dev, s_dev, b_dev, n, k, bits, group, int(interleave), C.byref(h)),
               "sd_qweight_create")
        self._h = h.value
        self.n, self.k = n, k

    def matmul(self, act_dev: int, m: int, y_dev: int, ldy: int, silu: bool = False, ws_dev: int | None = None,
               ws_bytes: int = 0, stream=None):
        _check(lib().sd_matmul(self._h, act_dev, m, y_dev, ldy, int(silu), ws_dev, ws_bytes, stream), "sd_matmul")

    def matmul_ex(self, act_dev: int, m: int, y_dev: int | None, ldy: int, silu: bool = False, x_dev: int | None = None,
                  ws_dev: int | None = None, ws_bytes: int = 0, algo: int = 0, stream=None):
        """`sd_matmul_ex`: algo 0 (the planner), 1 (tcgen05 tiles), 2 (the small-M kernel); with x_dev the
        f16-rounded products are added into the f32 rows at x_dev (ldy floats apart)."""
        _check(lib().sd_matmul_ex(self._h, act_dev, m, y_dev, ldy, int(silu), x_dev, ws_dev, ws_bytes, algo, stream),
               "sd_matmul")

    def __del__(self):
        try:
            if self._h:
                lib().sd_qweight_free(self._h)
        except Exception:
            pass


class NativeDecider:
    """The Decider of the library itself (`sd_decider_*`: tokenizer, prompt, torso, head and answers in
    C++), driven with System One JSON: `ask_all(request) -> response` as `Decider::evaluate` and
    `Response::to_json` (`src/lib.rs:46-87,147-150`)."""

    def __init__(self, handle: int):
        self._h = handle

    @classmethod
    def load(cls, model_dir: str, device: int = 0) -> "NativeDecider":
        h = C.c_void_p()
        if lib().sd_decider_load(os.fsencode(model_dir), device, C.byref(h)) != SD_OK:
            raise Error(f"Decider::load: {lib().sd_host_last_error().decode(errors='replace')}")
        return cls(h.value)

    def ask_all(self, request: dict) -> dict:
        out = C.c_void_p()
        L = lib()
        if L.sd_decider_ask_all(self._h, json.dumps(request).encode(), C.byref(out)) != SD_OK:
            raise Error(L.sd_decider_last_error(self._h).decode(errors="replace"))
        try:
            return json.loads(C.string_at(out.value).decode())
        finally:
            L.sd_string_free(out)

    def ask_batch(self, requests: list) -> list:
        """`sd_decider_ask_batch`: many requests at once (their states in packed passes, then all their
        questions in packed forks); a response body per request, or {"error": message}."""
        out = C.c_void_p()
        L = lib()
        if L.sd_decider_ask_batch(self._h, json.dumps(requests).encode(), C.byref(out)) != SD_OK:
            raise Error(L.sd_decider_last_error(self._h).decode(errors="replace"))
        try:
            return json.loads(C.string_at(out.value).decode())
        finally:
            L.sd_string_free(out)

    def close(self):
        if self._h:
            lib().sd_decider_free(self._h)
            self._h = None
