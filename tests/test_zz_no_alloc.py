"""kt_gs_radix_sort_pairs_static: the pair sort for callers that cannot allocate device memory
(a render loop with a fixed frame budget, a plugin whose host engine owns all device memory, a
process whose pool already holds the free memory). Its scratch is a fixed array inside the
library, so the test checks that two calls in a row - the second smaller than the first, over
the first call's leftovers - give exactly what the allocating entry point gives."""

import ctypes as C

import numpy as np
import pytest

from klartraum_b200 import _native as N

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

MAX_PAIRS = 1 << 20  # KT_GS_STATIC_SORT_MAX_PAIRS


def static_sort_fn():
    fn = N.load().kt_gs_radix_sort_pairs_static
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32, C.c_void_p]
    return fn


def make_pairs(n: int, key_bits: int, seed: int):
    rng = np.random.default_rng(seed)
    keys = rng.integers(0, 1 << 62, size=n, dtype=np.uint64) & np.uint64((1 << key_bits) - 1)
    keys[rng.integers(0, n, size=n // 4)] = keys[0]  # many equal keys: stability matters
    vals = rng.permutation(n).astype(np.uint32)
    return (torch.from_numpy(keys.view(np.int64)).cuda(), torch.from_numpy(vals.view(np.int32)).cuda())


def sort_allocating(kin, vin, n, key_bits):
    kout, vout = torch.empty_like(kin), torch.empty_like(vin)
    size = N.radix_sort_pairs(None, None, None, None, n, key_bits)
    temp = torch.empty(size, dtype=torch.uint8, device="cuda")
    N.radix_sort_pairs(kin, vin, kout, vout, n, key_bits, temp)
    torch.cuda.synchronize()
    return kout, vout


def sort_static(kin, vin, n, key_bits):
    kout, vout = torch.empty_like(kin), torch.empty_like(vin)
    st = static_sort_fn()(kin.data_ptr(), vin.data_ptr(), kout.data_ptr(), vout.data_ptr(), n, key_bits, None)
    assert st == N.KT_OK, N.STATUS_NAMES.get(st, st)
    torch.cuda.synchronize()
    return kout, vout


def test_static_sort_matches_allocating_sort_on_two_calls_in_a_row():
    for n, key_bits, seed in [(MAX_PAIRS, 45, 11), (300_001, 37, 12)]:
        kin, vin = make_pairs(n, key_bits, seed)
        k_ref, v_ref = sort_allocating(kin, vin, n, key_bits)
        k_st, v_st = sort_static(kin, vin, n, key_bits)
        assert torch.equal(k_st, k_ref) and torch.equal(v_st, v_ref)
        order = np.argsort(kin.cpu().numpy().view(np.uint64), kind="stable")
        assert np.array_equal(v_st.cpu().numpy(), vin.cpu().numpy()[order])


def test_static_sort_rejects_more_pairs_than_its_scratch_holds():
    kin, vin = make_pairs(16, 40, 3)
    st = static_sort_fn()(kin.data_ptr(), vin.data_ptr(), kin.data_ptr(), vin.data_ptr(), MAX_PAIRS + 1, 40, None)
    assert st == N.KT_ERR_CAPACITY
