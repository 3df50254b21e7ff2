"""kt_gs_radix_sort_pairs (the sort operator, GaussianSort in the reference) against a stable
numpy sort, including the reference test's known answer."""

import numpy as np
import pytest

from klartraum_b200 import native as N, reference_key

from helpers import load_kat

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def gpu_sort(keys: np.ndarray, vals: np.ndarray, key_bits: int):
    n = len(keys)
    kin = torch.from_numpy(keys.view(np.int64).copy()).cuda()
    vin = torch.from_numpy(vals.view(np.int32).copy()).cuda()
    kout = torch.empty_like(kin)
    vout = torch.empty_like(vin)
    size = N.radix_sort_pairs(None, None, None, None, n, key_bits)
    temp = torch.empty(max(size, 1), dtype=torch.uint8, device="cuda")
    N.radix_sort_pairs(kin, vin, kout, vout, n, key_bits, temp)
    torch.cuda.synchronize()
    assert torch.equal(kin.cpu(), torch.from_numpy(keys.view(np.int64)))  # input untouched
    return kout.cpu().numpy().view(np.uint64), vout.cpu().numpy().view(np.uint32)


def test_sort_known_answer():
    k = load_kat()["sort"]
    keys = reference_key(np.array(k["binMask"], np.uint64), np.array(k["z"], np.float32))
    sk, sv = gpu_sort(keys, np.arange(8, dtype=np.uint32), 64)
    assert list(sv) == k["expected_order"]
    assert np.all(np.diff(sk.astype(np.float64)) >= 0)


@pytest.mark.parametrize("n", [1, 2, 31, 4095, 4096, 4097, 100_000, 3_000_001])
@pytest.mark.parametrize("key_bits", [13, 37, 45, 64])
def test_sort_matches_stable_sort(n, key_bits):
    rng = np.random.default_rng(n * 131 + key_bits)
    mask = (1 << key_bits) - 1 if key_bits < 64 else (1 << 64) - 1
    keys = rng.integers(0, 1 << 63, size=n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, size=n, dtype=np.uint64)
    keys &= np.uint64(mask)
    if n > 100:
        keys[rng.integers(0, n, size=n // 3)] = keys[0]  # heavy ties
    vals = rng.permutation(n).astype(np.uint32)
    sk, sv = gpu_sort(keys, vals, key_bits)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(sk, keys[order])
    assert np.array_equal(sv, vals[order])


def test_sort_ignores_bits_above_key_bits():
    rng = np.random.default_rng(5)
    n = 50_000
    keys = rng.integers(0, 1 << 62, size=n, dtype=np.uint64)
    vals = np.arange(n, dtype=np.uint32)
    sk, sv = gpu_sort(keys, vals, 20)
    order = np.argsort(keys & np.uint64((1 << 20) - 1), kind="stable")
    assert np.array_equal(sv, vals[order])
    assert np.array_equal(sk, keys[order])


def test_sort_constant_and_zero_width_keys_are_stable_copies():
    n = 10_000
    keys = np.full(n, 77, np.uint64)
    vals = np.arange(n, dtype=np.uint32)[::-1].copy()
    for bits in (0, 8, 64):
        sk, sv = gpu_sort(keys, vals, bits)
        assert np.array_equal(sv, vals) and np.array_equal(sk, keys)


def test_sort_status_is_ok_after_a_sort_and_aliasing_is_refused():
    lib = N.load()
    n = 100_000
    rng = np.random.default_rng(9)
    kin = torch.from_numpy(rng.integers(0, 1 << 40, size=n, dtype=np.uint64).view(np.int64)).cuda()
    vin = torch.arange(n, dtype=torch.int32, device="cuda")
    kout, vout = torch.empty_like(kin), torch.empty_like(vin)
    size = N.radix_sort_pairs(None, None, None, None, n, 40)
    temp = torch.empty(size, dtype=torch.uint8, device="cuda")
    N.radix_sort_pairs(kin, vin, kout, vout, n, 40, temp)
    assert lib.kt_gs_radix_sort_status(temp.data_ptr(), None) == N.KT_OK
    # in place is refused before anything is enqueued
    with pytest.raises(N.KtError) as e:
        N.radix_sort_pairs(kin, vin, kin, vout, n, 40, temp)
    assert e.value.status == N.KT_ERR_ARG


def test_lookback_timeout_reaches_the_sort_status():
    """The bounded look-back wait of a sort pass, run against status words that nothing
    publishes (kt_gs_radix_sort_static_timeout_probe), gives up after its poll limit and records
    the timeout where a sort records it; kt_gs_radix_sort_status then reports KT_ERR_TIMEOUT, the
    context stays usable, and the next static sort clears the flag."""
    lib = N.load()
    assert lib.kt_gs_radix_sort_static_timeout_probe(0, None) == N.KT_ERR_ARG
    assert lib.kt_gs_radix_sort_static_timeout_probe(4096, None) == N.KT_OK
    assert lib.kt_gs_radix_sort_status(None, None) == N.KT_ERR_TIMEOUT
    n = 5000
    kin = torch.arange(n, 0, -1, dtype=torch.int64, device="cuda")
    vin = torch.arange(n, dtype=torch.int32, device="cuda")
    kout, vout = torch.empty_like(kin), torch.empty_like(vin)
    fn = lib.kt_gs_radix_sort_pairs_static
    import ctypes as C

    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32, C.c_void_p]
    assert fn(kin.data_ptr(), vin.data_ptr(), kout.data_ptr(), vout.data_ptr(), n, 16, None) == N.KT_OK
    assert lib.kt_gs_radix_sort_status(None, None) == N.KT_OK
    assert torch.equal(vout, torch.arange(n - 1, -1, -1, dtype=torch.int32, device="cuda"))
    assert fn(kin.data_ptr(), vin.data_ptr(), kin.data_ptr(), vout.data_ptr(), n, 16, None) == N.KT_ERR_ARG
