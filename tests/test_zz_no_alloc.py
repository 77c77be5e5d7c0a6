"""gf_sort_tile_keys_static: the tile-key sort for callers that cannot allocate
device memory while they render (under a host that gives the library a fixed
device budget and forbids allocation on its frame path).  It must return exactly the order
of the sort inside gf_tracer_trace, using only its fixed static scratch.

Collected last on purpose: a failure here leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest

from tests import harness

pytestmark = pytest.mark.gpu


def _traced_sort(device):
    """Sorted keys and ids of a real forward pass (the existing entry point),
    and the same pairs back in the order the tracer emits them (particle id,
    then tile index)."""
    from gofish_b200.scene import workload_cpu_scale

    w = workload_cpu_scale()
    case = harness.make_case(w.scene, w.camera, w.poses[0])
    gpu = harness.GpuTracer(case, 16, 0, device)
    got = gpu.forward()
    keys = got["keys"].view(np.uint64)
    ids = got["ids"].view(np.uint32)
    tiles = keys >> np.uint64(32)
    order = np.lexsort((tiles, ids))
    t = case.tmask.size
    end_bit = 32 + int(t).bit_length()
    return keys, ids, keys[order].copy(), ids[order].copy(), end_bit


def test_static_sort_matches_the_tracer_sort_on_two_consecutive_calls(cuda_device):
    import torch

    from gofish_b200 import _native

    lib = _native.load()
    sorted_keys, sorted_ids, emitted_keys, emitted_ids, end_bit = _traced_sort(cuda_device)
    n = sorted_keys.size
    assert 0 < n <= _native.STATIC_SORT_MAX_PAIRS
    keys_in = torch.from_numpy(emitted_keys.view(np.int64)).to(cuda_device)
    ids_in = torch.from_numpy(emitted_ids.view(np.int32)).to(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for call in range(2):
        keys_out = torch.full((n,), -1, dtype=torch.int64, device=cuda_device)
        ids_out = torch.full((n,), -1, dtype=torch.int32, device=cuda_device)
        code = lib.gf_sort_tile_keys_static(keys_in.data_ptr(), ids_in.data_ptr(), keys_out.data_ptr(),
                                            ids_out.data_ptr(), n, end_bit, stream)
        assert code == 0, lib.gf_last_error()
        torch.cuda.synchronize(cuda_device)
        np.testing.assert_array_equal(keys_out.cpu().numpy().view(np.uint64), sorted_keys, err_msg=f"call {call}")
        np.testing.assert_array_equal(ids_out.cpu().numpy().view(np.uint32), sorted_ids, err_msg=f"call {call}")
    # the inputs are read only
    np.testing.assert_array_equal(keys_in.cpu().numpy().view(np.uint64), emitted_keys)


def test_static_sort_rejects_more_pairs_than_its_scratch(cuda_device):
    from gofish_b200 import _native

    lib = _native.load()
    code = lib.gf_sort_tile_keys_static(None, None, None, None, _native.STATIC_SORT_MAX_PAIRS + 1, 46, None)
    assert code == -5  # GF_ERR_CAPACITY
    assert b"exceed the fixed scratch" in lib.gf_last_error()


def test_static_sort_at_its_limits(cuda_device):
    """MAX_PAIRS random keys (the whole histogram table, the grand total in its
    last slot) against a stable argsort; n = 0 and end_bit = 0 (nothing to
    sort: the pairs are copied)."""
    import torch

    from gofish_b200 import _native

    lib = _native.load()
    n = _native.STATIC_SORT_MAX_PAIRS
    rng = np.random.default_rng(17)
    keys = ((rng.integers(0, 4096, n, dtype=np.uint64) << np.uint64(32))
            | rng.integers(0, 1 << 20, n, dtype=np.uint64))  # repeated keys: stability matters
    ids = np.arange(n, dtype=np.uint32)
    order = np.argsort(keys, kind="stable")
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    k_in = torch.from_numpy(keys.view(np.int64)).to(cuda_device)
    i_in = torch.from_numpy(ids.view(np.int32)).to(cuda_device)
    k_out = torch.empty_like(k_in)
    i_out = torch.empty_like(i_in)
    assert lib.gf_sort_tile_keys_static(k_in.data_ptr(), i_in.data_ptr(), k_out.data_ptr(), i_out.data_ptr(), n, 44,
                                        stream) == 0, lib.gf_last_error()
    torch.cuda.synchronize(cuda_device)
    np.testing.assert_array_equal(k_out.cpu().numpy().view(np.uint64), keys[order])
    np.testing.assert_array_equal(i_out.cpu().numpy().view(np.uint32), ids[order])
    # end_bit 0: the pairs are copied in input order
    assert lib.gf_sort_tile_keys_static(k_in.data_ptr(), i_in.data_ptr(), k_out.data_ptr(), i_out.data_ptr(), 1000, 0,
                                        stream) == 0, lib.gf_last_error()
    torch.cuda.synchronize(cuda_device)
    np.testing.assert_array_equal(k_out.cpu().numpy()[:1000].view(np.uint64), keys[:1000])
    # n = 0: nothing is touched
    assert lib.gf_sort_tile_keys_static(None, None, None, None, 0, 44, stream) == 0, lib.gf_last_error()
