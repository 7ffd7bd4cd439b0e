"""The allocation-free bootstrap entry point (pnb_pbs_batch_noalloc).

Some callers cannot allocate GPU memory on the bootstrap path: their device memory is already
reserved by another framework's caching allocator, their request loop must not pay allocator
latency or synchronisation, or their FFI contract fixes the device footprint after start-up.
For them the library bootstraps into caller buffers using a fixed scratch array it holds for
the life of the process.  This test calls that entry point through the C ABI twice in a row,
with different batches, and checks each result word for word against pnb_pbs_batch on the same
inputs (both run the same deterministic kernels), and that a batch beyond the scratch limit is
refused.  It lives in its own file so that it runs after every other test.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_noalloc(pnb, keys, tv, ct, out):
    count = ct.shape[0]
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return pnb.lib().pnb_pbs_batch_noalloc(keys.handle, C.c_void_p(tv.data_ptr()),
                                           C.c_void_p(ct.data_ptr()), C.c_void_p(out.data_ptr()),
                                           count, stream)


def test_noalloc_bootstrap_matches_allocating_entry_point(pnb):
    keys = pnb.keygen(seed=31337, device=0)
    rng = np.random.default_rng(99)
    for call, count in enumerate((200, 37)):  # two calls in a row, different batches
        msgs = rng.integers(0, 16, count)
        lut = rng.integers(0, 16, 16)
        tv = pnb.test_vector(keys, lut)
        ct = pnb.encrypt(keys, torch.tensor(msgs), seed=1000 + call)
        want = pnb.pbs_batch(keys, tv, ct)
        got = torch.full_like(want, -1)
        rc = _call_noalloc(pnb, keys, tv, ct, got)
        assert rc == 0, pnb.lib().pnb_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: outputs differ"
        assert np.array_equal(pnb.decrypt_vec(keys, got).cpu().numpy(), lut[msgs])
    assert pnb.device_status(0) == 0


def test_noalloc_rejects_batches_beyond_the_scratch(pnb):
    keys = pnb.keygen(seed=31338, device=0)
    tv = pnb.test_vector(keys, list(range(16)))
    ct = pnb.encrypt(keys, torch.zeros(248, dtype=torch.int64), seed=5)
    out = torch.zeros_like(ct)
    rc = _call_noalloc(pnb, keys, tv, ct, out)
    assert rc == 1
    assert b"247" in pnb.lib().pnb_last_error()
    torch.cuda.synchronize()
    assert int(out.abs().sum().item()) == 0  # nothing ran
