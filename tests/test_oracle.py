"""The CPU oracle, pinned against golden vectors made by the reference's own
memmap loader (tests/golden/make_golden.py). CPU only."""
import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gather_golden.npz")


@pytest.fixture(scope="module")
def golden():
    oracle.build()
    z = np.load(GOLDEN)
    cases = {}
    for key in z.files:
        if "/" not in key:
            continue
        name, field = key.split("/", 1)
        cases.setdefault(name, {})[field] = z[key]
    return z, cases


def table_of(case):
    if int(case["kind"]) == 0:
        return case["table"]
    return oracle.synth_table(int(case["kind"]), int(case["seed"]), int(case["rows"]), int(case["cache_dim"]))


def same_bits(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype == b.dtype and a.view(np.uint8).tobytes() == b.view(np.uint8).tobytes()


def test_generator_pins(golden):
    z, _ = golden
    for s, e, v in z["synth_pins"]:
        assert oracle.synth_u64(int(s), int(e)) == int(v)


def test_generator_known_answers():
    # SplitMix64 seeded with 0: the first outputs of the published generator
    assert oracle.synth_u64(0, 0) == 0xE220A8397B1DCDAF
    assert oracle.synth_u64(0, 1) == 0x6E789E6AA1B965F4
    assert oracle.synth_u64(0, 2) == 0x06C45D188009454F


@pytest.mark.parametrize("name", ["homo_f32_d1024", "hetero_t0", "hetero_t1", "hetero_t2", "hetero_t3",
                                  "homo_f16_d768", "homo_f32_d128", "subset_d200_of_1024", "long_d512",
                                  "special_f32", "empty"])
def test_oracle_matches_reference_loader(golden, name):
    _, cases = golden
    c = cases[name]
    t = table_of(c)
    out = oracle.gather(t, c["ids"], dim=int(c["dim"]), key_off=int(c["key_off"]))
    assert same_bits(out, c["out"])


def test_planted_mistake_is_caught(golden):
    _, cases = golden
    c = cases["homo_f32_d1024"]
    out = oracle.gather(table_of(c), c["ids"], dim=int(c["dim"]))
    bad = out.copy()
    bad.view(np.uint32)[3, 17] ^= 1  # one flipped mantissa bit
    assert not same_bits(bad, c["out"])
    bad = out.copy()
    bad[[0, 1]] = bad[[1, 0]]  # two rows swapped
    assert not same_bits(bad, c["out"])


def test_special_values_are_bit_exact(golden):
    _, cases = golden
    c = cases["special_f32"]
    out = oracle.gather(c["table"], c["ids"])
    # NaN payloads and signed zeros survive (a float compare would not see them)
    assert same_bits(out, c["out"])
    assert np.isnan(out).any() and (np.signbit(out) & (out == 0)).any()


def test_mmap_index_select_matches_oracle(tmp_path):
    rows, cdim = 500, 256
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 9, rows, cdim)
    path = tmp_path / "feat.bin"
    t.tofile(path)
    mm = oracle.open_memmap_table(str(path), np.float32, rows, cdim)
    ids = np.random.default_rng(0).integers(0, rows - 3, size=77)
    ref = oracle.mmap_index_select(mm, ids, dim=100, key_off=3).numpy()
    assert same_bits(ref, oracle.gather(t, ids, dim=100, key_off=3))


@pytest.mark.parametrize("kind", [oracle.KIND_F32_UNIFORM, oracle.KIND_F16_BYTESUM, oracle.KIND_I64_RAW,
                                  oracle.KIND_F16_NORMAL])
def test_gather_synth_equals_table_gather(kind):
    rows, cdim, dim = 300, 96, 64
    t = oracle.synth_table(kind, 4, rows, cdim)
    ids = np.random.default_rng(1).integers(0, rows - 10, size=120)
    a = oracle.gather(t, ids, dim=dim, key_off=10)
    b = oracle.gather_synth(kind, 4, rows, cdim, dim, ids, key_off=10)
    assert same_bits(a, b)


def test_gather_synth_wrap():
    # element e holds synth(e mod wrap): equal to gathering ids mod wrap_rows when rows divide the wrap
    rows, cdim = 1000, 64
    wrap_rows = 128
    ids = np.random.default_rng(2).integers(0, rows, size=200)
    a = oracle.gather_synth(oracle.KIND_F32_UNIFORM, 6, rows, cdim, cdim, ids, wrap_elems=wrap_rows * cdim)
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 6, wrap_rows, cdim)
    assert same_bits(a, oracle.gather(t, ids % wrap_rows))


def test_out_of_range_ids_raise():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 10, 8)
    with pytest.raises(IndexError):
        oracle.gather(t, np.array([0, 10]))
    with pytest.raises(IndexError):
        oracle.gather(t, np.array([-1]))


def test_fp16_stream_is_exact_and_bell_shaped():
    t = oracle.synth_table(oracle.KIND_F16_BYTESUM, 1, 200, 768)
    v = t.astype(np.float64)
    # every value is a multiple of 2^-8 with |v| < 4
    assert np.all(np.abs(v) < 4.0)
    assert np.all((v * 256.0) == np.round(v * 256.0))
    assert abs(v.mean()) < 0.01 and 0.75 < v.std() < 0.9


def test_fp32_stream_is_uniform_grid():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 100, 1024).astype(np.float64)
    assert t.min() >= -1.0 and t.max() < 1.0
    assert np.all((t + 1.0) * 2**23 == np.round((t + 1.0) * 2**23))
    assert abs(t.mean()) < 0.01


def python_stripe(p, n, start, wrap):
    # page_cache_backup.h:626-652 (STRIPE): ctrl = p % n, device page = start + p / n
    q = p % wrap if wrap else p
    return q % n, start + q // n


@pytest.mark.parametrize("n,start,wrap", [(1, 0, 0), (4, 0, 0), (4, 7, 0), (3, 2, 0), (4, 0, 48), (8, 5, 64)])
def test_stripe_locate(n, start, wrap):
    for p in [0, 1, 2, 3, 5, 47, 48, 63, 64, 1000, 123456789]:
        assert oracle.stripe_locate(p, n, start, wrap) == python_stripe(p, n, start, wrap)


def test_stripe_image_round_trip():
    page = 512
    logical = np.arange(page * 37 // 4, dtype=np.uint32).view(np.uint8)
    devs = oracle.stripe_image(logical, page, 4, 3, (3 + 10) * page)
    back = np.zeros_like(logical)
    for p in range(37):
        c, dp = python_stripe(p, 4, 3, 0)
        back[p * page:(p + 1) * page] = devs[c][dp * page:(dp + 1) * page]
    assert np.array_equal(back, logical)


def test_fp16_normal_stream():
    """kind 4: normal(0, 1) by Box-Muller, rounded to fp16 (the config-4 features)."""
    t = oracle.synth_table(oracle.KIND_F16_NORMAL, 5, 400, 768)
    v = t.astype(np.float64)
    assert np.isfinite(v).all()
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01
    assert abs((np.abs(v) < 1.0).mean() - 0.6827) < 0.005 and abs((np.abs(v) < 2.0).mean() - 0.9545) < 0.003
    # element 0 of seed 5 by hand: the same transform in float64, rounded by numpy's float16 (RNE)
    h = int(oracle.synth_table(oracle.KIND_I64_RAW, 5, 1, 1).view(np.uint64)[0, 0])
    u1 = ((h >> 32) + 1.0) * 2.0 ** -32
    u2 = (h & 0xFFFFFFFF) * 2.0 ** -32
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2)
    assert np.float16(z).view(np.uint16) == t[0, 0].view(np.uint16)
