"""Python mirror of the reference's solve-service API over the C ABI.

The reference drives its GPU solver from Rust (engine/src/gpu/client.rs:
spawn / GpuClient::{submit, set_weights, queued_work} / SolveHandle::wait /
SolveResult; engine/src/serialize.rs: PackedJob). This module exposes the same
names and meanings over ``lib/libwcb200.so`` (include/wc_b200.h), so callers
and tests read like the reference's own. There is no CPU fallback: every
solve runs the CUDA kernels, and loading fails loudly if the library is
missing.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libwcb200.so")

WC_E_CAPPED = 3


class SolveError(RuntimeError):
    """A nonzero status from the C ABI (the reference's Err(String))."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class _SolveCfg(C.Structure):
    _fields_ = [("depth", C.c_int32), ("iters", C.c_int32), ("snapshots", C.c_int32), ("reserved", C.c_int32),
                ("alpha", C.c_float), ("beta", C.c_float), ("gamma", C.c_float), ("predict", C.c_float),
                ("node_cap", C.c_uint64)]


class _Weights(C.Structure):
    _fields_ = [("ndims", C.c_uint32), ("dims", C.POINTER(C.c_uint32)), ("w", C.c_void_p), ("nw", C.c_uint64),
                ("b", C.c_void_p), ("nb", C.c_uint64), ("ln", C.c_void_p), ("nln", C.c_uint64)]


class _JobInfo(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("nodes", "cells", "net_rows", "terminal_leaves", "configs", "levels",
                                          "root_nc0", "root_nc1", "ncarried", "carry_snapshots", "carry_width",
                                          "table_bytes")]


class _Result(C.Structure):
    _fields_ = [("strategy", C.POINTER(C.c_float)), ("ncells", C.c_uint64),
                ("root_values", C.POINTER(C.c_float)), ("nroots", C.c_uint64), ("root_width", C.c_uint64),
                ("carries", C.POINTER(C.c_uint16)), ("carry_snapshots", C.c_uint64), ("carry_width", C.c_uint64),
                ("weight_version", C.c_uint64), ("oversize_route", C.c_int32), ("card_exclusive_route", C.c_int32)]


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
    lib = C.CDLL(LIB_PATH)
    P, VP, U64, I = C.POINTER, C.c_void_p, C.c_uint64, C.c_int
    sig = {
        "wc_init": (I, [I, P(C.c_int), P(_Weights), I, P(VP)]),
        "wc_publish": (I, [VP, P(_Weights), P(U64)]),
        "wc_publish_device": (I, [VP, I, VP, VP, VP, P(U64)]),
        "wc_shutdown": (None, [VP]),
        "wc_last_error": (I, [C.c_char_p, C.c_size_t]),
        "wc_net_layout": (None, [P(U64), P(U64), P(U64)]),
        "wc_weights_fill": (I, [I, U64, VP, VP, VP]),
        "wc_set_cap_marker_value": (None, [C.c_float]),
        "wc_root_generate": (I, [U64, I, I, C.c_char_p, C.c_size_t, P(C.c_size_t)]),
        "wc_root_generate_wide": (I, [U64, I, I, C.c_uint32, C.c_char_p, C.c_size_t, P(C.c_size_t)]),
        "wc_job_build": (I, [C.c_char_p, C.c_size_t, P(_SolveCfg), VP, C.c_uint32, P(VP)]),
        "wc_job_build_batch": (I, [P(C.c_char_p), P(C.c_size_t), C.c_size_t, P(_SolveCfg), P(VP), P(C.c_uint32), I,
                                   P(VP), P(C.c_int)]),
        "wc_job_digest": (I, [VP, P(U64)]),
        "wc_job_info_get": (I, [VP, P(_JobInfo)]),
        "wc_job_free": (None, [VP]),
        "wc_job_root_belief": (I, [VP, VP]),
        "wc_job_counts": (I, [VP, P(U64), I]),
        "wc_job_carry_offsets": (I, [VP, VP, VP]),
        "wc_solve_batch": (I, [VP, P(VP), C.c_size_t, P(_Result)]),
        "wc_result_free": (None, [P(_Result)]),
        "wc_batch_upload": (I, [VP, I, P(VP), C.c_size_t, P(VP)]),
        "wc_batch_solve": (I, [VP]),
        "wc_batch_solve_profiled": (I, [VP, P(C.c_double), I]),
        "wc_batch_leaf_values": (I, [VP, I, P(C.c_double)]),
        "wc_batch_download_leaf_values": (I, [VP, C.c_size_t, I, VP]),
        "wc_batch_download_board_rows": (I, [VP, C.c_size_t, VP, VP]),
        "wc_batch_download": (I, [VP, C.c_size_t, VP, VP, VP]),
        "wc_batch_nash_conv": (I, [VP, VP, VP]),
        "wc_batch_stats": (None, [VP, P(C.c_double), P(C.c_double), P(U64), P(U64)]),
        "wc_batch_free": (None, [VP]),
        "wc_batch_launches": (U64, [VP]),
        "wc_submit": (I, [VP, VP, P(U64)]),
        "wc_wait": (I, [VP, U64, P(_Result)]),
        "wc_queued_work": (U64, [VP]),
        "wc_debug_umma_gemm": (I, [VP, VP, I, I, VP]),
        "wc_debug_umma_gemm_static": (I, [VP, VP, I, I, VP]),
        "wc_state_legal_actions": (I, [C.c_char_p, C.c_size_t, P(C.c_uint32), C.c_size_t, P(C.c_size_t)]),
        "wc_state_apply": (I, [C.c_char_p, C.c_size_t, C.c_uint32, I, C.c_char_p, C.c_size_t, P(C.c_size_t)]),
        "wc_state_query": (I, [C.c_char_p, C.c_size_t, P(C.c_int32)]),
        "wc_roots_file_split": (I, [C.c_char_p, C.c_size_t, P(U64), P(U64), C.c_size_t, P(C.c_size_t)]),
        "wc_game_new": (I, [U64, I, P(_SolveCfg), P(VP)]),
        "wc_game_from_root": (I, [C.c_char_p, C.c_size_t, U64, P(_SolveCfg), P(VP)]),
        "wc_game_set_max_solves": (I, [VP, C.c_uint32]),
        "wc_game_advance": (I, [VP, P(VP), P(C.c_int)]),
        "wc_game_resume": (I, [VP, VP, P(_Result)]),
        "wc_game_counters": (I, [VP, P(C.c_int64)]),
        "wc_game_root": (I, [VP, C.c_char_p, C.c_size_t, P(C.c_size_t)]),
        "wc_game_free": (None, [VP]),
        "wc_replay_pack_row": (I, [C.c_char_p, C.c_size_t, C.c_char_p]),
        "wc_wcj8_from_root": (I, [C.c_char_p, C.c_size_t, P(_SolveCfg), VP, C.c_uint32, P(C.c_uint32), C.c_uint32,
                                  C.c_char_p, C.c_size_t, P(C.c_size_t)]),
        "wc_job_from_wcj8": (I, [C.c_char_p, C.c_size_t, P(VP)]),
        "wc_debug_set_wait_limit": (I, [VP, U64]),
        "wc_replay_expand": (I, [VP, C.c_size_t, VP, VP, C.c_size_t, VP, VP, VP]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        buf = C.create_string_buffer(4096)
        lib().wc_last_error(buf, 4096)
        raise SolveError(rc, buf.value.decode(errors="replace"))


# ----------------------------------------------------------------- config

INF = float("inf")


@dataclass(frozen=True)
class Cfr:
    """The discounting rule (engine/src/search.rs:133-185)."""
    alpha: float
    beta: float
    gamma: float
    predict: float


Cfr.LINEAR = Cfr(1.0, 1.0, 1.0, 0.0)
Cfr.PLUS = Cfr(INF, -INF, 2.0, 0.0)
Cfr.DISCOUNTED = Cfr(1.5, 0.0, 2.0, 0.0)
Cfr.PREDICTIVE = Cfr(INF, -INF, 2.0, 1.0)
Cfr.SIMPLE_ASYM = Cfr(INF, -INF, 2.0, 1.0 / 3.0)
Cfr.NAMED = {"linear": Cfr.LINEAR, "plus": Cfr.PLUS, "dcfr": Cfr.DISCOUNTED, "pcfr": Cfr.PREDICTIVE,
             "sapcfr": Cfr.SIMPLE_ASYM}


@dataclass(frozen=True)
class Cfg:
    """search::Cfg (engine/src/search.rs:50-95)."""
    depth: int = 1
    iters: int = 64
    snapshots: bool = True
    cfr: Cfr = Cfr.LINEAR
    node_cap: int = 0

    def _c(self) -> _SolveCfg:
        return _SolveCfg(self.depth, self.iters, int(self.snapshots), 0, self.cfr.alpha, self.cfr.beta,
                         self.cfr.gamma, self.cfr.predict, self.node_cap)


def snapshot_iters(iters: int) -> List[int]:
    """Kept iterations: 0, the powers of two and the final one (search.rs:102-110)."""
    return [t for t in range(iters + 1) if t == 0 or (t & (t - 1)) == 0 or t == iters]


def set_cap_marker_value(v: float) -> None:
    lib().wc_set_cap_marker_value(v)


# ------------------------------------------------------------------ rules
# States travel in the reference's write_state encoding (engine/src/roots.rs:
# 150-180); action codes are Action::encode's (engine/src/actions.rs:252-295).

def legal_actions(state: bytes) -> List[int]:
    """State::legal_actions (engine/src/rules.rs:1027-1146): action codes in
    the engine's order."""
    codes = (C.c_uint32 * 512)()
    n = C.c_size_t()
    _check(lib().wc_state_legal_actions(state, len(state), codes, 512, C.byref(n)))
    return list(codes[: n.value])


def apply_action(state: bytes, code: int, unchecked: bool = False) -> bytes:
    """State::apply (engine/src/rules.rs:1155): the successor state's bytes.
    A non-legal action is refused unless `unchecked`, which applies it as the
    reference's apply does (no legality test; fields must still be in
    range)."""
    buf = C.create_string_buffer(4096)
    n = C.c_size_t()
    _check(lib().wc_state_apply(state, len(state), code, int(unchecked), buf, 4096, C.byref(n)))
    return buf.raw[: n.value]


ROW_BYTES = 215   # replay row (engine/src/rebel.rs:935-964)
PUBFEAT = 897     # the public encoding's width (engine/src/rebel.rs:1044)
CCOUNTS = 15      # config counts per config (engine/src/rebel.rs:68)


def pack_row(state: bytes) -> bytes:
    """pack_row (engine/src/rebel.rs:1236): the replay row of a state in the
    write_state encoding, or of the state a root starts with."""
    buf = C.create_string_buffer(ROW_BYTES)
    _check(lib().wc_replay_pack_row(state, len(state), buf))
    return buf.raw


def wcj8_bytes(root: bytes, cfg: "Cfg", carried: Optional[np.ndarray] = None, net_dims=(5,)) -> bytes:
    """PackedJob::from_solver(root's subgame, carried).to_bytes() (engine/src/
    serialize.rs:340-357, 1051-1125): the reference's WCJ8 job bytes."""
    if carried is not None:
        carried = np.ascontiguousarray(carried, np.float32)
        n, ptr = carried.shape[0], carried.ctypes.data
    else:
        n, ptr = 0, None
    dims = (C.c_uint32 * max(1, len(net_dims)))(*net_dims)
    need = C.c_size_t()
    rc = lib().wc_wcj8_from_root(root, len(root), C.byref(cfg._c()), ptr, n, dims, len(net_dims), None, 0,
                                 C.byref(need))
    if rc != 1 or need.value == 0:
        _check(rc)
    buf = C.create_string_buffer(need.value)
    _check(lib().wc_wcj8_from_root(root, len(root), C.byref(cfg._c()), ptr, n, dims, len(net_dims), buf,
                                   need.value, C.byref(need)))
    return buf.raw[: need.value]


def state_query(state: bytes) -> dict:
    """to_act, winner (None while undecided), is_terminal, is_chance."""
    out = (C.c_int32 * 4)()
    _check(lib().wc_state_query(state, len(state), out))
    return {"to_act": out[0], "winner": None if out[1] < 0 else out[1], "terminal": bool(out[2]),
            "chance": bool(out[3])}


def split_roots_file(data: bytes) -> List[bytes]:
    """The roots of a version-3 roots file (roots::read_roots,
    engine/src/roots.rs:337-363), each in the root encoding wc_job_build
    takes."""
    n = C.c_size_t()
    cap = max(1, len(data) // 16)
    off = (C.c_uint64 * cap)()
    ln = (C.c_uint64 * cap)()
    _check(lib().wc_roots_file_split(data, len(data), off, ln, cap, C.byref(n)))
    return [data[off[i]: off[i] + ln[i]] for i in range(n.value)]


def generate_root(seed: int, plies: int = 20, random_draft: bool = True) -> bytes:
    """A seeded solve-site root: State bytes and both beliefs."""
    cap = 1 << 20
    buf = C.create_string_buffer(cap)
    n = C.c_size_t()
    _check(lib().wc_root_generate(seed, plies, int(random_draft), buf, cap, C.byref(n)))
    return buf.raw[: n.value]


def generate_wide_root(seed: int, ncfg: int = 256, plies: int = 20, random_draft: bool = True) -> bytes:
    """A belief-heavy root: generate_root's position
    with each player's belief over up to ncfg consistent configs, Dirichlet(1)
    weights (wc_root_generate_wide)."""
    cap = 1 << 22
    buf = C.create_string_buffer(cap)
    n = C.c_size_t()
    _check(lib().wc_root_generate_wide(seed, plies, int(random_draft), ncfg, buf, cap, C.byref(n)))
    return buf.raw[: n.value]


# ---------------------------------------------------------------- weights

def net_layout():
    w, b, l = C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib().wc_net_layout(C.byref(w), C.byref(b), C.byref(l))
    return w.value, b.value, l.value


def seeded_weights(kind: str = "he", seed: int = 0):
    """(dims, w, b, ln) for the v5 blob: "he" (seeded He-normal) or "test"
    (the reference GPU tests' blob, engine/src/gpu/tests.rs:34-48)."""
    nw, nb, nl = net_layout()
    w = np.zeros(nw, np.float32)
    b = np.zeros(nb, np.float32)
    ln = np.zeros(nl, np.float32)
    k = {"he": 0, "test": 1}[kind]
    _check(lib().wc_weights_fill(k, seed, w.ctypes.data, b.ctypes.data, ln.ctypes.data))
    return [5], w, b, ln


def _weights_struct(dims, w, b, ln):
    if w is None:
        return None, None
    d = (C.c_uint32 * len(dims))(*dims)
    ws = _Weights(len(dims), d, w.ctypes.data, w.size, b.ctypes.data, b.size, ln.ctypes.data, ln.size)
    return ws, (d, w, b, ln)


# ------------------------------------------------------------------- jobs

class PackedJob:
    """One subgame solve (engine/src/serialize.rs:143-150), flattened."""

    def __init__(self, handle: int, root: bytes, cfg: Cfg):
        self._h = C.c_void_p(handle)
        self.root = root
        self.cfg = cfg
        info = _JobInfo()
        _check(lib().wc_job_info_get(self._h, C.byref(info)))
        self.info = {n: getattr(info, n) for n, _ in _JobInfo._fields_}

    @classmethod
    def from_root(cls, root: bytes, cfg: Cfg, carried: Optional[np.ndarray] = None) -> "PackedJob":
        h = C.c_void_p()
        if carried is not None:
            carried = np.ascontiguousarray(carried, np.float32)
            n = carried.shape[0]
            ptr = carried.ctypes.data
        else:
            n, ptr = 0, None
        _check(lib().wc_job_build(root, len(root), C.byref(cfg._c()), ptr, n, C.byref(h)))
        return cls(h.value, root, cfg)

    @classmethod
    def from_wcj8(cls, data: bytes, cfg: Cfg) -> "PackedJob":
        """A job from the reference's WCJ8 job bytes (PackedJob::from_bytes,
        engine/src/serialize.rs:1127); `cfg` records the solve configuration
        the bytes carry."""
        h = C.c_void_p()
        _check(lib().wc_job_from_wcj8(data, len(data), C.byref(h)))
        return cls(h.value, b"", cfg)

    @classmethod
    def build_many(cls, roots: Sequence[bytes], cfg: Cfg, threads: int = 0,
                   carried: Optional[Sequence[Optional[np.ndarray]]] = None) -> List[Optional["PackedJob"]]:
        """Jobs for many roots on native host threads (wc_job_build_batch): the
        parallel form of the reference tape builder (wave_tape.rs:48-61).
        carried[i], if given, is root i's carried root pairs as in from_root.
        A root whose tree hits the node cap gives None, as the tape builder
        skips it; any other failure raises."""
        n = len(roots)
        arr = (C.c_char_p * n)(*roots)
        lens = (C.c_size_t * n)(*[len(r) for r in roots])
        out = (C.c_void_p * n)()
        status = (C.c_int * n)()
        cptr, ncar, keep = None, None, []
        if carried is not None:
            cptr, ncar = (C.c_void_p * n)(), (C.c_uint32 * n)()
            for i, c in enumerate(carried):
                if c is not None:
                    c = np.ascontiguousarray(c, np.float32)
                    keep.append(c)
                    cptr[i], ncar[i] = c.ctypes.data, c.shape[0]
        rc = lib().wc_job_build_batch(arr, lens, n, C.byref(cfg._c()), cptr, ncar, threads, out, status)
        jobs = [cls(out[i], roots[i], cfg) if out[i] else None for i in range(n)]
        _check(rc)
        return jobs

    @property
    def digest(self) -> int:
        """64-bit digest of the flattened tables (wc_job_digest)."""
        d = C.c_uint64()
        _check(lib().wc_job_digest(self._h, C.byref(d)))
        return d.value

    def counts(self) -> np.ndarray:
        """Per-player work counts (see wc_job_counts)."""
        out = (C.c_uint64 * 21)()
        _check(lib().wc_job_counts(self._h, out, 21))
        return np.array(list(out), np.int64)

    def root_belief(self) -> np.ndarray:
        """Both players' root weights, player 0 first."""
        out = np.zeros(self.info["root_nc0"] + self.info["root_nc1"], np.float32)
        _check(lib().wc_job_root_belief(self._h, out.ctypes.data))
        return out

    def carry_layout(self):
        """(offsets over the exit nodes, exit node ids) of a carry row."""
        n = self.info["net_rows"] + self.info["terminal_leaves"]
        off = np.zeros(n + 1, np.uint32)
        ids = np.zeros(max(n, 1), np.uint32)
        _check(lib().wc_job_carry_offsets(self._h, off.ctypes.data, ids.ctypes.data))
        return off, ids[:n]

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.wc_job_free(self._h)
            self._h = C.c_void_p()


@dataclass
class SolveResult:
    """engine/src/gpu/client.rs:115-122."""
    strategy: np.ndarray
    root_values: List[List[np.ndarray]]
    carries: Optional[np.ndarray]
    weight_version: int
    oversize_route: bool = False
    card_exclusive_route: bool = False


def _take_result(r: _Result, job: PackedJob) -> SolveResult:
    strat = np.ctypeslib.as_array(r.strategy, (r.ncells,)).copy() if r.ncells else np.zeros(0, np.float32)
    n0 = job.info["root_nc0"]
    roots = np.ctypeslib.as_array(r.root_values, (r.nroots * r.root_width,)).copy().reshape(r.nroots, r.root_width)
    rv = [[row[:n0].copy(), row[n0:].copy()] for row in roots]
    carries = None
    if r.carry_snapshots:
        carries = np.ctypeslib.as_array(r.carries, (r.carry_snapshots * r.carry_width,)).copy().view(np.float16)
        carries = carries.reshape(r.carry_snapshots, r.carry_width)
    out = SolveResult(strat, rv, carries, r.weight_version, bool(r.oversize_route), bool(r.card_exclusive_route))
    lib().wc_result_free(C.byref(r))
    return out


# ---------------------------------------------------------------- service

class SolveHandle:
    def __init__(self, client: "GpuClient", ticket: int, job: PackedJob):
        self._client, self._ticket, self._job = client, ticket, job

    def wait(self) -> SolveResult:
        r = _Result()
        _check(lib().wc_wait(self._client._ctx, self._ticket, C.byref(r)))
        return _take_result(r, self._job)


class GpuClient:
    """engine/src/gpu/client.rs: submit / set_weights / queued_work."""

    def __init__(self, ctx: int):
        self._ctx = C.c_void_p(ctx)

    def submit(self, job: PackedJob) -> SolveHandle:
        t = C.c_uint64()
        _check(lib().wc_submit(self._ctx, job._h, C.byref(t)))
        return SolveHandle(self, t.value, job)

    def set_weights(self, dims, w, b, ln) -> int:
        ws, keep = _weights_struct(dims, w, b, ln)
        v = C.c_uint64()
        _check(lib().wc_publish(self._ctx, C.byref(ws) if ws else None, C.byref(v)))
        return v.value

    def set_weights_device(self, dev_index: int, w_ptr: int, b_ptr: int, ln_ptr: int) -> int:
        v = C.c_uint64()
        _check(lib().wc_publish_device(self._ctx, dev_index, w_ptr, b_ptr, ln_ptr, C.byref(v)))
        return v.value

    def queued_work(self) -> int:
        return lib().wc_queued_work(self._ctx)

    def solve_batch(self, jobs: Sequence[PackedJob]) -> List[SolveResult]:
        n = len(jobs)
        arr = (C.c_void_p * n)(*[j._h.value for j in jobs])
        res = (_Result * n)()
        _check(lib().wc_solve_batch(self._ctx, arr, n, res))
        return [_take_result(res[i], jobs[i]) for i in range(n)]

    def play(self, games: Sequence["Game"], threads: Optional[int] = None,
             stats: Optional[dict] = None) -> int:
        """Drive games to their end (the reference's GPU game stream,
        selfplay.rs:1224: game actors building subgames while the GPU
        service batches whatever they have submitted).

        Each game advances to its next solve on one of `threads` host
        threads on its own: tree build and flattening. The default is the
        cores divided among the node's ranks (LOCAL_WORLD_SIZE, as torchrun
        sets it; 1 without it).
        Whenever the device is idle, every subgame ready at that moment is
        solved in one wc_solve_batch. Each game then resumes its walk with its
        own result, on the calling thread between solves, so its job's pinned
        tables are released while the device is idle, and its next build
        starts at once. A subgame's solve does not depend on the batch it
        lands in, so the games play exactly as one at a time would. A build
        error is raised here once the builds in flight have finished.
        Returns the subgames solved; `stats`, when given, receives the
        batches, the largest batch, the solved subgames' nodes and the
        seconds spent in wc_solve_batch."""
        import queue
        import time
        from concurrent.futures import ThreadPoolExecutor

        games = list(games)
        ready: "queue.Queue" = queue.Queue()  # (game, job or None when the game is over, error)

        def build(g):
            try:
                ready.put((g, g.advance(), None))
            except BaseException as e:  # handed to the solving thread, which raises it
                ready.put((g, None, e))

        solved = batches = biggest = nodes = 0
        solve_s = 0.0
        if not threads:
            threads = (os.cpu_count() or 1) // max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1") or 1))
        pool = ThreadPoolExecutor(max(1, threads))
        try:
            for g in games:
                pool.submit(build, g)
            active = len(games)
            while active:
                got = [ready.get()]   # block until a subgame (or a finished game) is ready
                while True:           # then take everything else ready now
                    try:
                        got.append(ready.get_nowait())
                    except queue.Empty:
                        break
                pend = []
                for g, job, err in got:
                    if err is not None:
                        raise err
                    if job is None:
                        active -= 1
                    else:
                        pend.append((g, job))
                del got
                if not pend:
                    continue
                n = len(pend)
                arr = (C.c_void_p * n)(*[j._h.value for _, j in pend])
                res = (_Result * n)()
                t0 = time.perf_counter()
                _check(lib().wc_solve_batch(self._ctx, arr, n, res))
                solve_s += time.perf_counter() - t0
                try:
                    for i, (g, j) in enumerate(pend):
                        _check(lib().wc_game_resume(g._h, j._h, C.byref(res[i])))
                finally:
                    for i in range(n):
                        lib().wc_result_free(C.byref(res[i]))
                for g, _ in pend:
                    pool.submit(build, g)
                solved += n
                batches += 1
                biggest = max(biggest, n)
                nodes += sum(j.info["nodes"] for _, j in pend)
                del pend, arr, res
        finally:
            pool.shutdown(wait=True, cancel_futures=True)
        if stats is not None:
            stats.update(batches=batches, largest_batch=biggest, nodes=nodes, solve_s=solve_s)
        return solved

    def upload(self, jobs: Sequence[PackedJob], dev_index: int = 0) -> "DeviceBatch":
        n = len(jobs)
        arr = (C.c_void_p * n)(*[j._h.value for j in jobs])
        h = C.c_void_p()
        _check(lib().wc_batch_upload(self._ctx, dev_index, arr, n, C.byref(h)))
        return DeviceBatch(h.value, list(jobs))

    def close(self) -> None:
        if self._ctx.value:
            lib().wc_shutdown(self._ctx)
            self._ctx = C.c_void_p()


class DeviceBatch:
    """A batch resident on one device: solve repeatedly, read back per job."""

    def __init__(self, handle: int, jobs: List[PackedJob]):
        self._h = C.c_void_p(handle)
        self.jobs = jobs

    def solve(self) -> None:
        _check(lib().wc_batch_solve(self._h))

    TIME_CLASSES = ["net_solve", "leaf", "rows", "vgather", "reach", "snapshot", "phase2", "init", "total",
                    "pool", "join", "head", "trunk"]

    def solve_profiled(self) -> dict:
        """One solve with per-class CUDA-event timings (ms) on the runtime's stream."""
        ms = (C.c_double * 13)()
        _check(lib().wc_batch_solve_profiled(self._h, ms, len(ms)))
        return dict(zip(self.TIME_CLASSES, list(ms)))

    def leaf_values(self, p: int, profile: bool = False):
        """Run leaf evaluation alone for traverser p (initial reaches); with
        profile=True return the per-class timings in ms."""
        ms = (C.c_double * 13)() if profile else None
        _check(lib().wc_batch_leaf_values(self._h, p, ms))
        return dict(zip(self.TIME_CLASSES, list(ms))) if profile else None

    def leaf_values_of(self, j: int, p: int) -> np.ndarray:
        n = int(self.jobs[j].counts()[14 + p])
        out = np.zeros(max(n, 1), np.float32)
        _check(lib().wc_batch_download_leaf_values(self._h, j, p, out.ctypes.data))
        return out[:n]

    def board_rows(self, j: int):
        """(P[rows, 256], jp[rows, 128]) of job j as the network path stores them."""
        n = self.jobs[j].info["net_rows"]
        pb = np.zeros((max(n, 1), 256), np.float32)
        jp = np.zeros((max(n, 1), 128), np.float32)
        _check(lib().wc_batch_download_board_rows(self._h, j, pb.ctypes.data, jp.ctypes.data))
        return pb[:n], jp[:n]

    def nash_conv(self):
        """After solve(): per job (nash_conv, zero_sum) of the average strategy
        from the live root belief (Solver::nash_conv, search.rs:1884-1907),
        computed on the device."""
        n = len(self.jobs)
        nash = np.zeros(max(n, 1), np.float32)
        zs = np.zeros(max(n, 1), np.float32)
        _check(lib().wc_batch_nash_conv(self._h, nash.ctypes.data, zs.ctypes.data))
        return nash[:n], zs[:n]

    def launches(self) -> int:
        """Kernel launches of the last solve or leaf evaluation."""
        return int(lib().wc_batch_launches(self._h))

    def stats(self):
        nu, le = C.c_double(), C.c_double()
        tb, db = C.c_uint64(), C.c_uint64()
        lib().wc_batch_stats(self._h, C.byref(nu), C.byref(le), C.byref(tb), C.byref(db))
        return {"node_updates": nu.value, "leaf_evals": le.value, "table_bytes": tb.value, "device_bytes": db.value}

    def result(self, j: int) -> SolveResult:
        job = self.jobs[j]
        info = job.info
        strat = np.zeros(info["cells"], np.float32)
        width = info["root_nc0"] + info["root_nc1"]
        roots = np.zeros(info["ncarried"] * width, np.float32)
        carries = np.zeros(max(info["carry_snapshots"] * info["carry_width"], 1), np.uint16)
        _check(lib().wc_batch_download(self._h, j, strat.ctypes.data, roots.ctypes.data, carries.ctypes.data))
        roots = roots.reshape(info["ncarried"], width)
        n0 = info["root_nc0"]
        c = None
        if info["carry_snapshots"]:
            c = carries[: info["carry_snapshots"] * info["carry_width"]].view(np.float16)
            c = c.reshape(info["carry_snapshots"], info["carry_width"])
        return SolveResult(strat, [[r[:n0].copy(), r[n0:].copy()] for r in roots], c, 0)

    def free(self) -> None:
        if self._h.value:
            lib().wc_batch_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        if getattr(self, "_h", None) is not None and self._h.value and _lib is not None:
            self.free()


class Game:
    """A game of two solving seats with continual re-solving (selfplay.rs:
    466-905 Game::advance / resume): advance() plays to the next subgame
    solve and returns its job (or None when the game is over); the caller
    solves it and calls resume(job, result) (GpuClient.play drives many games
    this way)."""

    COUNTERS = ["decisions", "solves", "capped", "walk_decisions", "walk_draws", "ended", "winner", "walking"]

    def __init__(self, cfg: Cfg, seed: int = 0, random_draft: bool = True, root: Optional[bytes] = None,
                 max_solves: int = 0):
        self.cfg = cfg
        h = C.c_void_p()
        if root is None:
            _check(lib().wc_game_new(seed, int(random_draft), C.byref(cfg._c()), C.byref(h)))
        else:
            _check(lib().wc_game_from_root(root, len(root), seed, C.byref(cfg._c()), C.byref(h)))
        self._h = h
        if max_solves:
            _check(lib().wc_game_set_max_solves(self._h, max_solves))

    def advance(self) -> Optional[PackedJob]:
        job, step = C.c_void_p(), C.c_int()
        _check(lib().wc_game_advance(self._h, C.byref(job), C.byref(step)))
        return PackedJob(job.value, b"", self.cfg) if step.value == 1 else None

    def counters(self) -> dict:
        out = (C.c_int64 * 8)()
        _check(lib().wc_game_counters(self._h, out))
        return dict(zip(self.COUNTERS, list(out)))

    def root(self) -> bytes:
        """The current state and beliefs in the root encoding."""
        n = C.c_size_t()
        buf = C.create_string_buffer(1 << 22)
        _check(lib().wc_game_root(self._h, buf, 1 << 22, C.byref(n)))
        return buf.raw[: n.value]

    def __del__(self):
        if getattr(self, "_h", None) is not None and self._h.value and _lib is not None:
            lib().wc_game_free(self._h)
            self._h = C.c_void_p()


NET_MODES = {"bf16": 0, "exact": 1, "f16": 2}


def spawn(device, dims=None, w=None, b=None, ln=None, precise: bool = True, net: Optional[str] = None) -> GpuClient:
    """gpu::service::spawn (engine/src/gpu/service.rs:55-82). `device` is an
    index or a list of indices; w=None runs without a value network.

    net: "exact" (fp32, the reference CPU network's operation order), "f16"
    or "bf16" (tcgen05 tensor cores with that operand type, fp32 accumulate).
    Without `net`, precise=True means "exact" and False means "f16" (the
    reference GPU service's fast mode computes with f16 operands)."""
    mode = NET_MODES[net if net is not None else ("exact" if precise else "f16")]
    devs = [device] if isinstance(device, int) else list(device)
    arr = (C.c_int * len(devs))(*devs)
    ws, keep = _weights_struct(dims, w, b, ln)
    h = C.c_void_p()
    _check(lib().wc_init(len(devs), arr, C.byref(ws) if ws else None, mode, C.byref(h)))
    return GpuClient(h.value)


def debug_umma_gemm(a_bf16: np.ndarray, b_bf16: np.ndarray) -> np.ndarray:
    """tcgen05 self-test: A[128, K] @ B[N, K]^T with bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(a_bf16, np.uint16)
    b = np.ascontiguousarray(b_bf16, np.uint16)
    k, n = a.shape[1], b.shape[0]
    d = np.zeros((128, n), np.float32)
    _check(lib().wc_debug_umma_gemm(a.ctypes.data, b.ctypes.data, k, n, d.ctypes.data))
    return d
