"""The library's host-side topology (wavefront_nd.h, wavefront_plan.h,
km_topology.h) against the reference: golden plans built by the reference
C sources, the known answers of tests/unit/test_wavefront_nd.c, and the
oracle on random shapes.  Integer results must be bit-exact."""
import ctypes as C

import numpy as np
import pytest

import kmamba_b200 as kb

i64 = np.int64


def arr(v):
    return np.ascontiguousarray(v, dtype=i64)


def plan_arrays(lib, dims):
    d = arr(dims)
    pl = lib.km_wavefront_plan_create(d.ctypes.data, len(dims))
    assert pl
    c = pl.contents
    ls = np.ctypeslib.as_array(c.level_starts, (c.max_level + 2,)).copy()
    lo = np.ctypeslib.as_array(c.level_offsets, (c.total_points,)).copy()
    meta = (c.total_points, c.max_level, c.max_level_size)
    assert lib.km_wavefront_plan_matches_dims(pl, d.ctypes.data, len(dims)) == 1
    for lvl in range(c.max_level + 1):
        assert lib.km_wavefront_plan_level_size(pl, lvl) == ls[lvl + 1] - ls[lvl]
    assert lib.km_wavefront_plan_level_size(pl, c.max_level + 1) == -1
    assert not lib.km_wavefront_plan_level_offsets(pl, -1)
    lib.km_wavefront_plan_free(pl)
    return ls, lo, meta


def test_plans_bitexact_vs_reference_golden(lib, golden):
    for tag, g in golden("plans.npz").items():
        ls, lo, meta = plan_arrays(lib, g["dims"])
        np.testing.assert_array_equal(ls, g["level_starts"], err_msg=tag)
        np.testing.assert_array_equal(lo, g["level_offsets"], err_msg=tag)
        assert tuple(meta) == tuple(g["meta"]), tag


@pytest.mark.parametrize("seed", range(8))
def test_plans_vs_oracle_random(lib, oracle, seed):
    rng = np.random.default_rng(seed)
    nd = int(rng.integers(1, 6))
    dims = rng.integers(1, 9, nd)
    ls, lo, _ = plan_arrays(lib, dims)
    ols, olo = oracle.wavefront_plan(dims)
    np.testing.assert_array_equal(ls, ols)
    np.testing.assert_array_equal(lo, olo)
    for lvl in range(len(ls) - 1):
        assert lib.wavefront_nd_level_size(arr(dims).ctypes.data, nd, lvl) == ls[lvl + 1] - ls[lvl]


def test_level_sizes_known_answers(lib):
    # tests/unit/test_wavefront_nd.c:104-160
    d = arr([3, 4])
    assert lib.wavefront_nd_max_level(d.ctypes.data, 2) == 5
    assert [lib.wavefront_nd_level_size(d.ctypes.data, 2, i) for i in range(6)] == \
        [1, 2, 3, 3, 2, 1]
    d = arr([2, 3, 2])
    assert lib.wavefront_nd_max_level(d.ctypes.data, 3) == 4
    assert [lib.wavefront_nd_level_size(d.ctypes.data, 3, i) for i in range(5)] == \
        [1, 3, 4, 3, 1]
    assert lib.wavefront_nd_level_size(d.ctypes.data, 3, 5) == -1
    assert lib.wavefront_nd_row_major_offset(d.ctypes.data, arr([1, 2, 1]).ctypes.data, 3) == 11
    assert lib.wavefront_nd_row_major_offset(d.ctypes.data, arr([2, 0, 0]).ctypes.data, 3) == -1


def test_full_coverage_and_ordinal_order(lib):
    # tests/unit/test_wavefront_nd.c:162-210
    d = arr([2, 3, 2])
    seen = []

    @kb.VISIT_FN
    def visit(idx, ndims, level, ordinal, user):
        co = [idx[i] for i in range(ndims)]
        assert sum(co) == level
        if seen and seen[-1][0] == level:
            assert ordinal == seen[-1][1] + 1
        else:
            assert ordinal == 0
        seen.append((level, ordinal, co))
        return 0

    assert lib.wavefront_nd_for_each_level(d.ctypes.data, 3, None, visit, None) == 0
    offs = [lib.wavefront_nd_row_major_offset(d.ctypes.data, arr(c).ctypes.data, 3)
            for _, _, c in seen]
    assert sorted(offs) == list(range(12))
    # inside a level: lexicographic (= ascending row-major) order
    for lvl in range(5):
        lv = [o for (L, _, _), o in zip(seen, offs) if L == lvl]
        assert lv == sorted(lv)


def test_early_stop(lib):
    # tests/unit/test_wavefront_nd.c:212-232: the callback's code is returned
    d = arr([3, 4])
    count = [0]

    @kb.VISIT_FN
    def visit(idx, ndims, level, ordinal, user):
        count[0] += 1
        return 77 if count[0] >= 2 else 0

    assert lib.wavefront_nd_for_level(d.ctypes.data, 2, 3, None, visit, None) == 77
    assert count[0] == 2
    scratch = arr([0, 0])
    count[0] = 0
    assert lib.wavefront_nd_for_level(d.ctypes.data, 2, 3, scratch.ctypes.data, visit, None) == 77


def test_invalid_params(lib):
    # tests/unit/test_wavefront_nd.c:234-248
    bad = arr([3, 0])

    @kb.VISIT_FN
    def visit(*a):
        return 0

    assert lib.wavefront_nd_validate_dims(bad.ctypes.data, 2) == 0
    assert lib.wavefront_nd_total_points(bad.ctypes.data, 2) == -1
    assert lib.wavefront_nd_max_level(bad.ctypes.data, 2) == -1
    assert lib.wavefront_nd_for_each_level(bad.ctypes.data, 2, None, visit, None) == -1
    assert not lib.km_wavefront_plan_create(bad.ctypes.data, 2)
    assert lib.wavefront_nd_validate_dims(None, 2) == 0
    assert lib.wavefront_nd_validate_dims(arr([4]).ctypes.data, 0) == 0
    huge = arr([1 << 40, 1 << 40])
    assert lib.wavefront_nd_total_points(huge.ctypes.data, 2) == -1


def test_km_topology_helpers(lib):
    d = arr([3, 4, 5])
    st = arr([0, 0, 0])
    assert lib.km_make_row_major_strides(d.ctypes.data, 3, st.ctypes.data) == 1
    assert list(st) == [20, 5, 1]
    co = arr([0, 0, 0])
    for lin in range(60):
        lib.km_unravel_index(lin, d.ctypes.data, st.ctypes.data, 3, co.ctypes.data)
        assert lib.km_ravel_index(co.ctypes.data, d.ctypes.data, st.ctypes.data, 3) == lin
    assert lib.km_ravel_index(arr([3, 0, 0]).ctypes.data, d.ctypes.data, st.ctypes.data, 3) == -1
    assert lib.km_power_long(3, 4) == 81
    assert lib.km_power_long(0, 0) == 0
    assert lib.km_power_long(2, -1) == 0
    prod = C.c_size_t(0)
    assert lib.km_spatial_dims_product(d.ctypes.data, 3, C.byref(prod)) == 1
    assert prod.value == 60
    assert lib.km_spatial_dims_product(d.ctypes.data, 9, C.byref(prod)) == 0
    # km_normalize_spatial_topology: implicit 1D topology
    nd = arr([0])
    dims = arr([0] * 8)
    cnd = arr([0])
    assert lib.km_normalize_spatial_topology(nd.ctypes.data, dims.ctypes.data, 128, 1,
                                             cnd.ctypes.data, 3) == 0
    assert nd[0] == 1 and dims[0] == 128 and cnd[0] == 1
    nd = arr([2])
    dims = arr([8, 16] + [0] * 6)
    assert lib.km_normalize_spatial_topology(nd.ctypes.data, dims.ctypes.data, 128, 0,
                                             None, 0) == 0
    assert lib.km_normalize_spatial_topology(nd.ctypes.data, dims.ctypes.data, 100, 0,
                                             None, 0) == -1
    cnd = arr([3])
    assert lib.km_normalize_spatial_topology(nd.ctypes.data, dims.ctypes.data, 128, 1,
                                             cnd.ctypes.data, 3) == -1


def test_convnd_kernel_volume(lib):
    assert lib.convnd_kernel_volume(2, 3) == 9
    assert lib.convnd_kernel_volume(3, 3) == 27
    assert lib.convnd_kernel_volume(0, 3) == 0
    assert lib.convnd_kernel_volume(2, 0) == 0
