"""The allocation-free histogram entry point (mojotrees_b200_histogram_u8_noalloc).

Callers that cannot allocate GPU memory -- applications whose pool allocator
owns the device, latency-critical paths that must not take allocator locks --
get the same histogram as mojotrees_b200_histogram_u8 from device buffers they
own, with the library's fixed device array as the only scratch.  This file is
collected last so that a stop-at-first-failure run has already run every
other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(seed, n, F, B):
    rng = np.random.default_rng(seed)
    bins = rng.integers(0, B, size=(F, n), dtype=np.uint8)
    g = rng.integers(-2, 3, size=n).astype(np.int8)
    h = rng.integers(0, 5, size=n).astype(np.uint8)
    rows = np.sort(rng.choice(n, size=n // 3, replace=False)).astype(np.int32)
    return bins, g, h, rows


def _noalloc(mtlib, bins, B, g, h, rows):
    import torch
    F, n = bins.shape
    Fp = (F + 15) // 16 * 16
    rm = np.zeros((n, Fp), np.uint8)
    rm[:, :F] = bins.T
    pairs = (g.view(np.uint8)[rows].astype(np.uint16) | (h[rows].astype(np.uint16) << 8)).view(np.int16)
    d_bins = torch.from_numpy(rm).cuda()
    d_rows = torch.from_numpy(rows).cuda()
    d_pairs = torch.from_numpy(pairs.copy()).cuda()
    d_out = torch.full((F, 3, B), -7, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    lib = mtlib.lib()
    e = lib.mojotrees_error_create()
    try:
        rc = lib.mojotrees_b200_histogram_u8_noalloc(d_bins.data_ptr(), n, F, B, d_rows.data_ptr(), rows.size,
                                                    d_pairs.data_ptr(), 4, d_out.data_ptr(),
                                                    ctypes.c_void_p(stream.cuda_stream), e)
        msg = lib.mojotrees_error_message(e).decode()
    finally:
        lib.mojotrees_error_free(e)
    assert rc == 0, msg
    torch.cuda.synchronize()
    return d_out.cpu().numpy()


def test_noalloc_matches_allocating_entry_twice(mtlib):
    # two calls in a row; the second is smaller, so stale cells from the
    # first call would show up if the shared array were not cleared
    for seed, n, F, B in ((1, 120_000, 100, 255), (2, 30_000, 40, 63)):
        bins, g, h, rows = _inputs(seed, n, F, B)
        want = mtlib.histogram_u8(bins, B, g, h, rows=rows)
        got = _noalloc(mtlib, bins, B, g, h, rows)
        np.testing.assert_array_equal(got, want)


def test_noalloc_rejects_sizes_beyond_the_array(mtlib):
    lib = mtlib.lib()
    e = lib.mojotrees_error_create()
    rc = lib.mojotrees_b200_histogram_u8_noalloc(1, 10, 200, 255, 1, 5, 1, 4, 1, None, e)
    msg = lib.mojotrees_error_message(e).decode()
    lib.mojotrees_error_free(e)
    assert rc == -1 and "allocation-free limit" in msg
