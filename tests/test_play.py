"""GpuClient.play's host loop on the CPU (the reference's GPU game stream,
selfplay.rs:1224): the library calls that need a device are faked, the loop
is the package's own. Games build on host threads, each batch holds what was
ready, every game reaches its solve limit with one resume per solve, no game
is advanced by two threads at once, and a build failure is raised."""
import ctypes as C
import random
import threading
import time

import pytest


class Job:
    made = 0

    def __init__(self):
        Job.made += 1
        self._h = C.c_void_p(Job.made)
        self.info = {"nodes": 10}


class FakeGame:
    """Seeded, uneven build times; refuses concurrent advances."""

    def __init__(self, seed, solves, fail_at=None):
        self.rng, self.left, self.fail_at = random.Random(seed), solves, fail_at
        self._h = C.c_void_p(seed + 1)
        self.busy = threading.Lock()
        self.resumed = 0

    def advance(self):
        assert self.busy.acquire(blocking=False), "a game advanced by two threads at once"
        try:
            time.sleep(self.rng.random() * 0.01)
            if self.left == self.fail_at:
                raise RuntimeError("planted build failure")
            if self.left == 0:
                return None
            self.left -= 1
            return Job()
        finally:
            self.busy.release()


class FakeCalls:
    def __init__(self, games):
        self.games = {g._h.value: g for g in games}
        self.batches, self.freed = [], 0

    def wc_solve_batch(self, ctx, arr, n, res):
        self.batches.append(n)
        time.sleep(0.005)
        return 0

    def wc_game_resume(self, g, j, r):
        self.games[g.value].resumed += 1
        return 0

    def wc_result_free(self, r):
        self.freed += 1
        return 0


def play(wc, monkeypatch, games, threads=4):
    calls = FakeCalls(games)
    monkeypatch.setattr(wc, "lib", lambda: calls)
    stats = {}
    solved = wc.GpuClient(0).play(games, threads=threads, stats=stats)
    return solved, stats, calls


def test_play_solves_every_game_to_its_limit(wc, monkeypatch):
    games = [FakeGame(s, solves=8) for s in range(12)]
    solved, stats, calls = play(wc, monkeypatch, games)
    assert solved == 96 and sum(calls.batches) == 96 and calls.freed == 96
    assert all(g.resumed == 8 and g.left == 0 for g in games)
    assert stats["batches"] == len(calls.batches) and stats["largest_batch"] == max(calls.batches)
    assert stats["nodes"] == 960 and stats["solve_s"] > 0
    assert max(calls.batches) <= 12 and len(calls.batches) >= 8


def test_play_with_games_that_end_at_once(wc, monkeypatch):
    games = [FakeGame(s, solves=0) for s in range(3)] + [FakeGame(9, solves=2)]
    solved, stats, calls = play(wc, monkeypatch, games, threads=1)
    assert solved == 2 and games[-1].resumed == 2


def test_play_raises_a_build_failure(wc, monkeypatch):
    games = [FakeGame(s, solves=6, fail_at=2 if s == 3 else None) for s in range(6)]
    with pytest.raises(RuntimeError, match="planted"):
        play(wc, monkeypatch, games)
