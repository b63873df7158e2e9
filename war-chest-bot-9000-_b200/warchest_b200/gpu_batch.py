"""Device-side expansion of compact replay rows for the trainer: the same
interface as the reference's train/gpu_batch.py (make_batch, warmup), with
the expansion in this library's CUDA kernel (wc_replay_expand) instead of a
Triton kernel. torch holds the device buffers and supplies the stream.

make_batch(parts, rng, device) takes the replay buffer's compact batch
(rows, aux, cc, cp, cw, cy, seg) and returns, on `device`, what the CPU
batch (train/train.py:249-270) returns: (x [2n, PUBFEAT], phi [m, 15],
weights, seg, targets, owner, 2n). View 2r of x is row r, view 2r + 1 its
board mirror with the seats exchanged (train/mirror.py:60-85); the sizes
of each view's seats come from the first config of its (row, seat) span.
"""
import numpy as np

from . import CCOUNTS, PUBFEAT, ROW_BYTES, SolveError, _check, lib


def _spans_ok(seg: np.ndarray, n: int) -> bool:
    """Every (row, seat) span 0 .. 2n - 1 present, in order: the CPU batch's
    np.searchsorted lookup (train/train.py:75) needs each to start inside
    the config arrays."""
    if seg.ndim != 1 or (len(seg) and np.any(np.diff(seg) < 0)):
        return False
    starts = np.searchsorted(seg, np.arange(2 * n, dtype=np.int64), side="left")
    return bool(np.all(starts < len(seg)))


def make_batch(parts, rng, device):
    """Compact replay batch -> two canonical query rows per replay row, on
    `device` (a CUDA device); `rng` is unused, as in the reference."""
    import torch

    del rng
    rows, aux, cc, cp, cw, cy, seg = parts
    rows = np.ascontiguousarray(rows, np.uint8).reshape(-1, ROW_BYTES)
    cc = np.ascontiguousarray(cc, np.uint8).reshape(-1, CCOUNTS)
    seg = np.ascontiguousarray(seg, np.int64)
    n, m = len(rows), len(cc)
    if len(seg) != m:
        raise SolveError(1, "seg and cc differ in length")
    if not _spans_ok(seg, n):
        raise SolveError(1, "seg must be non-decreasing with every span 2 row + seat present")
    device = torch.device(device)
    t = lambda a, dtype: torch.as_tensor(a, dtype=dtype, device=device)
    rows_t = t(rows, torch.uint8)
    cc_t = t(cc, torch.uint8)
    seg_t = t(seg, torch.long)
    x = torch.empty((2 * n, PUBFEAT), dtype=torch.float32, device=device)
    phi = torch.empty((m, CCOUNTS), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        _check(lib().wc_replay_expand(rows_t.data_ptr(), n, cc_t.data_ptr(), seg_t.data_ptr(), m, x.data_ptr(),
                                      phi.data_ptr(), stream))
    return (x, phi, t(cw, torch.float32), seg_t, t(cy, torch.float32), t(aux, torch.int64), 2 * n)


def warmup(device):
    """Load the kernel and its tables before the run's wall clock starts."""
    import torch

    rows = np.zeros((1, ROW_BYTES), np.uint8)
    cc = np.zeros((2, CCOUNTS), np.uint8)
    parts = (rows, np.zeros((1, 10), np.uint8), cc, np.asarray([0, 1], np.uint8), np.ones(2, np.float32),
             np.zeros(2, np.float32), np.asarray([0, 1], np.int64))
    make_batch(parts, None, device)
    torch.cuda.synchronize(device)
