"""ctypes access to the CPU oracle (oracle/_build/liboracle.so).

Test infrastructure only: the oracle restates the reference solver
(engine/src/search.rs) and value network (engine/src/net.rs) on the CPU and
is the checker for the CUDA path.
"""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_PATH = os.path.join(ROOT, "oracle", "_build", "liboracle.so")


class OCfg(C.Structure):
    _fields_ = [("depth", C.c_int32), ("iters", C.c_int32), ("snapshots", C.c_int32), ("pad", C.c_int32),
                ("alpha", C.c_float), ("beta", C.c_float), ("gamma", C.c_float), ("predict", C.c_float),
                ("node_cap", C.c_uint64)]


_lib = None


def _weight_ptrs(weights):
    """The weight arrays as pointers. Entry points without declared argument
    types receive a Python int as a 32-bit C int, which cuts an address above
    4 GB, so every pointer goes through c_void_p."""
    if weights is None:
        return None, None, None
    _, wa, ba, la = weights
    return C.c_void_p(wa.ctypes.data), C.c_void_p(ba.ctypes.data), C.c_void_p(la.ctypes.data)


def lib():
    global _lib
    if _lib is None:
        L = C.CDLL(ORACLE_PATH)
        VP = C.c_void_p
        L.oracle_solver_new.restype = VP
        L.oracle_solver_new.argtypes = [C.c_char_p, C.c_size_t, C.POINTER(OCfg), VP, VP, VP]
        for n in ["oracle_solver_free", "oracle_solver_multistep", "oracle_solver_shape", "oracle_root_sizes",
                  "oracle_nash_conv", "oracle_value_under", "oracle_carried_beliefs", "oracle_solver_snapshot",
                  "oracle_net_pieces", "oracle_exit_leaves"]:
            getattr(L, n).argtypes = None
        L.oracle_solver_ncells.restype = C.c_size_t
        L.oracle_solver_ncells.argtypes = [VP]
        L.oracle_solver_nsnaps.restype = C.c_size_t
        L.oracle_solver_nsnaps.argtypes = [VP]
        L.oracle_exit_leaves.restype = C.c_size_t
        L.oracle_solver_outcomes.argtypes = [VP]
        L.oracle_tabular_value.restype = C.c_double
        L.oracle_tabular_value.argtypes = [C.c_char_p, C.c_size_t, C.c_int]
        L.oracle_last_error.restype = C.c_char_p
        L.oracle_set_cap_marker_value.argtypes = [C.c_float]
        L.oracle_solve_many.argtypes = [C.POINTER(C.c_char_p), C.POINTER(C.c_size_t), C.c_size_t,
                                        C.POINTER(OCfg), VP, VP, VP, C.c_int, C.POINTER(C.c_double)]
        L.oracle_leaf_values.restype = C.c_size_t
        L.oracle_leaf_values.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.oracle_bench.argtypes = [C.POINTER(C.c_char_p), C.POINTER(C.c_size_t), C.c_size_t, C.POINTER(OCfg),
                                   VP, VP, VP, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]
        _lib = L
    return _lib


def ocfg(cfg):
    """oracle config from a warchest_b200.Cfg."""
    c = cfg.cfr
    return OCfg(cfg.depth, cfg.iters, int(cfg.snapshots), 0, c.alpha, c.beta, c.gamma, c.predict, cfg.node_cap)


class Oracle:
    """The reference solver on one root (search.rs Solver)."""

    def __init__(self, root: bytes, cfg, weights=None):
        self.cfg = cfg
        self._keep = weights
        w, b, ln = _weight_ptrs(weights)
        self.h = C.c_void_p(lib().oracle_solver_new(root, len(root), C.byref(ocfg(cfg)), w, b, ln))
        if not self.h.value:
            raise RuntimeError(lib().oracle_last_error().decode())
        s = (C.c_uint64 * 7)()
        lib().oracle_solver_shape(self.h, s)
        self.shape = dict(zip(["nodes", "cells", "net_rows", "terminal_leaves", "configs", "levels", "all_terminal"],
                              list(s)))
        rs = (C.c_uint64 * 2)()
        lib().oracle_root_sizes(self.h, rs)
        self.nc0, self.nc1 = rs[0], rs[1]

    def multistep(self, iters: int) -> None:
        lib().oracle_solver_multistep(self.h, C.c_int(iters))

    def snapshot(self, which: int = -1) -> np.ndarray:
        n = lib().oracle_solver_nsnaps(self.h)
        if which < 0:
            which += n
        out = np.zeros(lib().oracle_solver_ncells(self.h), np.float32)
        lib().oracle_solver_snapshot(self.h, C.c_size_t(which), out.ctypes.data_as(C.c_void_p))
        return out

    def nsnaps(self) -> int:
        return lib().oracle_solver_nsnaps(self.h)

    def value_under(self, roots: np.ndarray) -> np.ndarray:
        roots = np.ascontiguousarray(roots, np.float32)
        out = np.zeros_like(roots)
        lib().oracle_value_under(self.h, roots.ctypes.data_as(C.c_void_p), C.c_size_t(roots.shape[0]),
                                 out.ctypes.data_as(C.c_void_p))
        return out

    def nash_conv(self):
        n, z = C.c_float(), C.c_float()
        lib().oracle_nash_conv(self.h, C.byref(n), C.byref(z))
        return n.value, z.value

    def set_strategy(self, strategy: np.ndarray) -> None:
        """Evaluate an external average strategy (reference cell layout) in
        nash_conv / value_under from now on."""
        s = np.ascontiguousarray(strategy, np.float32)
        if lib().oracle_set_strategy(self.h, s.ctypes.data_as(C.c_void_p), C.c_size_t(s.size)):
            raise ValueError("strategy length does not match the tree")

    def exit_leaves(self) -> np.ndarray:
        n = lib().oracle_exit_leaves(self.h, None)
        out = np.zeros(n, np.uint32)
        lib().oracle_exit_leaves(self.h, out.ctypes.data_as(C.c_void_p))
        return out

    def carried_beliefs(self, leaf: int, width: int) -> np.ndarray:
        n = self.nsnaps() - 1
        out = np.zeros(max(n, 1) * width, np.float32)
        lib().oracle_carried_beliefs(self.h, C.c_uint32(leaf), out.ctypes.data_as(C.c_void_p))
        return out[: n * width].reshape(n, width)

    def leaf_values(self, p: int) -> np.ndarray:
        """Network-row values for traverser p at the current reaches
        (search.rs:1550 leaf_values), rows in leaf_rows order."""
        L = lib()
        n = L.oracle_leaf_values(self.h, p, None)
        out = np.zeros(max(n, 1), np.float32)
        L.oracle_leaf_values(self.h, p, out.ctypes.data_as(C.c_void_p))
        return out[:n]

    def net_pieces(self):
        s = self.shape
        pb = np.zeros(s["net_rows"] * 256, np.float32)
        jp = np.zeros(s["net_rows"] * 128, np.float32)
        f = np.zeros(s["configs"] * 256, np.float32)
        g = np.zeros(s["configs"] * 64, np.float32)
        rc = lib().oracle_net_pieces(self.h, pb.ctypes.data_as(C.c_void_p), jp.ctypes.data_as(C.c_void_p),
                                     f.ctypes.data_as(C.c_void_p), g.ctypes.data_as(C.c_void_p))
        if rc:
            raise RuntimeError("oracle has no network")
        return pb.reshape(-1, 256), jp.reshape(-1, 128), f.reshape(-1, 256), g.reshape(-1, 64)

    def __del__(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().oracle_solver_free(self.h)
            self.h = C.c_void_p()


def walk(seed: int, cfg, weights=None, max_solves: int = 0, random_draft: bool = True):
    """The continual re-solving game with every subgame solved by the CPU
    solver (oracle_walk): (counters dict, final root bytes)."""
    w, b, ln = _weight_ptrs(weights)
    ctr = (C.c_int64 * 8)()
    buf = C.create_string_buffer(1 << 22)
    n = C.c_size_t()
    rc = lib().oracle_walk(C.c_uint64(seed), int(random_draft), C.byref(ocfg(cfg)), w, b, ln, C.c_uint32(max_solves),
                           ctr, buf, C.c_size_t(1 << 22), C.byref(n))
    if rc:
        raise RuntimeError(lib().oracle_last_error().decode())
    names = ["decisions", "solves", "capped", "walk_decisions", "walk_draws", "ended", "winner", "walking"]
    return dict(zip(names, list(ctr))), buf.raw[: n.value]


def micro_root(seed: int, warmup: int, plies: int):
    buf = C.create_string_buffer(1 << 20)
    n = C.c_size_t()
    rc = lib().oracle_micro_root(C.c_uint64(seed), warmup, plies, buf, C.c_size_t(1 << 20), C.byref(n))
    return buf.raw[: n.value] if rc == 0 else None


def tabular_value(root: bytes, iters: int = 100) -> float:
    return lib().oracle_tabular_value(root, len(root), iters)


def solve_many(roots, cfg, weights, threads: int) -> float:
    """Solve every root on `threads` host threads; returns node-updates."""
    n = len(roots)
    arr = (C.c_char_p * n)(*roots)
    lens = (C.c_size_t * n)(*[len(r) for r in roots])
    out = C.c_double()
    w, b, ln = _weight_ptrs(weights)
    lib().oracle_solve_many(arr, lens, n, C.byref(ocfg(cfg)), w, b, ln, threads, C.byref(out))
    return out.value


def bench(roots, cfg, weights, threads: int, k1: int = 2, k2: int = 4):
    """Bounded CPU baseline (see oracle_bench): (node-updates/s, wall s, subgames)."""
    n = len(roots)
    arr = (C.c_char_p * n)(*roots)
    lens = (C.c_size_t * n)(*[len(r) for r in roots])
    out = (C.c_double * 3)()
    w, b, ln = _weight_ptrs(weights)
    lib().oracle_bench(arr, lens, n, C.byref(ocfg(cfg)), w, b, ln, threads, k1, k2, out)
    return out[0], out[1], int(out[2])
