"""gs3d_sort_pairs_no_alloc (static device scratch, no temp storage) against the existing
gs3d_sort_pairs_async entry point, both through the C ABI. Collected last (file name), so the
first call on the device may come either from this file alone or after every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

import gs3d
from gs3d import _abi

pytestmark = pytest.mark.gpu

MAX_ITEMS = 1 << 20  # GS3D_SORT_NO_ALLOC_MAX_ITEMS


def _inputs(n, seed):
    rng = np.random.default_rng(seed)
    keys = rng.integers(0, 1 << 62, n, dtype=np.int64)
    keys[: n // 3] = keys[n // 2]  # runs of equal keys: stability matters
    vals = rng.permutation(n).astype(np.int32)
    return keys, vals


def _sort_existing(lib, k_in, v_in, n, bits):
    k_out, v_out = torch.empty_like(k_in), torch.empty_like(v_in)
    nbytes = lib.determine_sort_pairs_temp_storage(None, None, None, None, n, bits)
    tmp = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=k_in.device)
    _abi.check(lib.gs3d_sort_pairs_async(C.c_void_p(tmp.data_ptr()), nbytes,
                                         C.c_void_p(k_in.data_ptr()), C.c_void_p(k_out.data_ptr()),
                                         C.c_void_p(v_in.data_ptr()), C.c_void_p(v_out.data_ptr()),
                                         n, bits, None))
    return k_out, v_out


def _sort_no_alloc(lib, k_in, v_in, n, bits, stream=None):
    k_out, v_out = torch.empty_like(k_in), torch.empty_like(v_in)
    rc = lib.gs3d_sort_pairs_no_alloc(C.c_void_p(k_in.data_ptr()), C.c_void_p(k_out.data_ptr()),
                                      C.c_void_p(v_in.data_ptr()), C.c_void_p(v_out.data_ptr()),
                                      n, bits, stream)
    _abi.check(rc)
    return k_out, v_out


def test_two_calls_in_a_row_match_the_existing_entry_point(cuda):
    """Two back-to-back calls on one stream share the static scratch: a full-size call, then a
    smaller one with a different bit width, whose result must not see the first's leftovers."""
    lib = gs3d.lib()
    cases = [(MAX_ITEMS, 46, 1), (300_007, 41, 2)]
    ins, outs = [], []
    for n, bits, seed in cases:
        keys, vals = _inputs(n, seed)
        ins.append((torch.from_numpy(keys).to(cuda), torch.from_numpy(vals).to(cuda)))
    torch.cuda.synchronize()
    for (k_in, v_in), (n, bits, _) in zip(ins, cases):
        outs.append(_sort_no_alloc(lib, k_in, v_in, n, bits))  # no sync between the two calls
    torch.cuda.synchronize()
    for (k_in, v_in), (n, bits, seed), (ko, vo) in zip(ins, cases, outs):
        rk, rv = _sort_existing(lib, k_in, v_in, n, bits)
        torch.cuda.synchronize()
        assert torch.equal(ko, rk) and torch.equal(vo, rv), (n, bits)
        keys, vals = _inputs(n, seed)
        assert np.array_equal(k_in.cpu().numpy(), keys)  # inputs untouched


def test_small_and_boundary_sizes(cuda):
    lib = gs3d.lib()
    # (1000, 0): no key bits, the sort only copies; (MAX_ITEMS, 64): the widest keys at the limit
    for n, bits in [(1, 35), (4095, 64), (4096, 33), (4097, 8), (1000, 0), (MAX_ITEMS, 64)]:
        keys, vals = _inputs(n, n + bits)
        k_in, v_in = torch.from_numpy(keys).to(cuda), torch.from_numpy(vals).to(cuda)
        ko, vo = _sort_no_alloc(lib, k_in, v_in, n, bits)
        rk, rv = _sort_existing(lib, k_in, v_in, n, bits)
        torch.cuda.synchronize()
        assert torch.equal(ko, rk) and torch.equal(vo, rv), (n, bits)


def test_zero_items_and_oversize_are_handled_without_launching(cuda):
    lib = gs3d.lib()
    assert lib.gs3d_sort_pairs_no_alloc(None, None, None, None, 0, 40, None) == 0
    k = torch.zeros(8, dtype=torch.int64, device=cuda)
    v = torch.zeros(8, dtype=torch.int32, device=cuda)
    # an oversize count is rejected before any pointer is touched (the buffers are tiny)
    rc = lib.gs3d_sort_pairs_no_alloc(C.c_void_p(k.data_ptr()), C.c_void_p(k.data_ptr()),
                                      C.c_void_p(v.data_ptr()), C.c_void_p(v.data_ptr()),
                                      MAX_ITEMS + 1, 40, None)
    assert rc == -1
    msg = lib.gs3d_last_error_string().decode()
    assert "exceeds the fixed scratch limit" in msg and str(MAX_ITEMS) in msg
    assert lib.gs3d_sort_pairs_no_alloc(None, None, None, None, -3, 40, None) == -1
