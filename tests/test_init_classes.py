"""init / cleanup / gpuName / getDevice / getAdapter / isBenchmarkEnabled and the
GpuMatrix / GpuVector classes, ported from the reference's own tests
(tests/init/src/test.init.js:30-200, tests/utils/test.classes.js:104-300;
complex types are outside this build's scope). The init semantics run on CPU
over the stand-in library (tests/fake_native.py: two fake devices), which
keeps the module-level device cache private to each test; the class tests run
there and on a B200 through the real library. The two-device example
(examples/init-two-gpus/init-two-gpus.js) runs on two GPUs when there are two."""
from __future__ import annotations

import threading
import warnings

import numpy as np
import pytest

from fake_native import FakeLib


@pytest.fixture()
def rt(wg, monkeypatch):
    """A clean runtime over the fake library; the real cache is restored afterwards."""
    from wgblas_b200 import _native as nat
    from wgblas_b200 import _runtime

    fake = FakeLib(nat.lib)
    monkeypatch.setattr(nat, "lib", fake)
    monkeypatch.setattr(_runtime, "_devices", {})
    monkeypatch.setattr(_runtime, "_primary", None)
    monkeypatch.delenv("WGBLAS_CUDA_DEVICES", raising=False)
    yield wg, fake


# ---- tests/init/src/test.init.js --------------------------------------------

def test_get_device_and_adapter_throw_before_init(rt):
    wg, _ = rt
    with pytest.raises(wg.Error, match=r"call init\(\) first"):
        wg.getDevice()
    with pytest.raises(wg.Error, match=r"call init\(\) first"):
        wg.getAdapter()
    with pytest.raises(wg.Error, match=r"call init\(\) first"):
        wg.gpuName()


def test_is_benchmark_enabled_false_for_unregistered_device(rt):
    wg, _ = rt
    assert wg.isBenchmarkEnabled({"label": "never-from-init"}) is False
    assert wg.isBenchmarkEnabled() is False


def test_first_init_with_dump_shaders_builds_a_working_device(rt):
    wg, _ = rt
    with warnings.catch_warnings(record=True):
        warnings.simplefilter("always")
        dev = wg.init(dumpShaders=True)
    assert dev is not None and wg.gpuName(dev)["description"]


def test_repeat_init_with_identical_options_returns_the_same_device(rt):
    wg, fake = rt
    first = wg.init()
    assert wg.init() is first
    assert fake.opened == 1


def test_differing_options_yield_a_distinct_device(rt):
    wg, _ = rt
    plain = wg.init()
    bench = wg.init(benchmark=True)
    assert bench is not plain
    assert wg.init() is plain and wg.init(benchmark=True) is bench
    assert wg.isBenchmarkEnabled(bench) and not wg.isBenchmarkEnabled(plain)
    assert not wg.isBenchmarkEnabled()  # the primary is the first one


def test_get_device_returns_the_primary_and_get_adapter_its_adapter(rt):
    wg, _ = rt
    first = wg.init()
    wg.init(benchmark=True)
    assert wg.getDevice() is first
    assert wg.getAdapter() is first.adapter is wg.getAdapter(first)
    assert wg.getAdapter().info["architecture"] == "sm_100"


def test_gpu_name_defaults_to_the_first_init(rt):
    wg, _ = rt
    first = wg.init()
    assert wg.gpuName() == wg.gpuName(first)
    assert wg.gpuName()["description"] and wg.gpuName()["device"] == "Fake B200"


def test_gpu_name_falls_back_to_unknown(rt):
    wg, _ = rt
    dev = wg.init()
    adapter = wg.getAdapter(dev)
    original = adapter.info
    adapter.info = {"device": "", "description": ""}
    try:
        assert wg.gpuName(dev) == {"description": "unknown", "device": "unknown"}
    finally:
        adapter.info = original


def test_cleanup_releases_every_cached_device(rt):
    wg, fake = rt
    wg.init()
    wg.init(benchmark=True)
    wg.cleanup()
    assert fake.closed == 2
    with pytest.raises(wg.Error, match=r"call init\(\) first"):
        wg.gpuName()
    fresh = wg.init()
    assert fresh is not None and wg.getDevice() is fresh


def test_cleanup_of_one_device_releases_only_that_device(rt):
    wg, _ = rt
    plain = wg.init()
    bench = wg.init(benchmark=True)
    wg.cleanup(bench)
    assert wg.init() is plain
    assert wg.gpuName(plain)["description"]
    with pytest.raises(wg.Error):
        wg.gpuName(bench)
    rebuilt = wg.init(benchmark=True)
    assert rebuilt is not bench


def test_cleanup_promotes_a_survivor_to_primary(rt):
    wg, _ = rt
    plain = wg.init()
    bench = wg.init(benchmark=True)
    assert wg.gpuName() == wg.gpuName(plain)
    wg.cleanup(plain)
    assert wg.getDevice() is bench
    assert wg.gpuName() == wg.gpuName(bench)
    wg.cleanup(bench)
    with pytest.raises(wg.Error):
        wg.getDevice()


def test_cleanup_of_unknown_or_released_device_is_a_no_op(rt):
    wg, fake = rt
    dev = wg.init()
    wg.cleanup({"not": "a device"})
    wg.cleanup(dev)
    wg.cleanup(dev)
    assert fake.closed == 1


def test_power_preference_picks_two_devices(rt):
    """examples/init-two-gpus/init-two-gpus.js: high-performance and low-power land
    on different GPUs when there are two (first and last ordinal)."""
    wg, _ = rt
    d_gpu = wg.init(powerPreference="high-performance")
    i_gpu = wg.init(powerPreference="low-power")
    assert (d_gpu.ordinal, i_gpu.ordinal) == (0, 1)
    assert wg.gpuName(d_gpu)["description"] != wg.gpuName(i_gpu)["description"]


# ---- tests/utils/test.classes.js: GpuMatrix / GpuVector ------------------------

BACKENDS = ["fake", pytest.param("gpu", marks=pytest.mark.gpu)]


@pytest.fixture(params=BACKENDS)
def cls(request, wg):
    """(wg, device) on the fake library or on the real one (the session's GPU device)."""
    if request.param == "fake":
        rt_ = request.getfixturevalue("rt")
        return rt_[0], rt_[0].init()
    return wg, request.getfixturevalue("device")


def test_matrix_round_trips_dense_float32(cls):
    wg, dev = cls
    m = wg.GpuMatrix.from_(dev, np.array([1, 2, 3, 4], np.float32), 2, 2)
    back = m.read()
    m.destroy()
    assert back.dtype == np.float32 and back.tolist() == [1, 2, 3, 4]


@pytest.mark.parametrize("layout", ["row-major", "column-major"])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_matrix_strips_lda_padding(cls, layout, dt):
    wg, dev = cls
    m = wg.GpuMatrix.from_(dev, np.array([1, 2, 0, 3, 4, 0], dt), 2, 2, 3, layout)
    back = m.read()
    m.destroy()
    assert back.dtype == dt and back.tolist() == [1, 2, 3, 4]


def test_matrix_round_trips_float64_exactly(cls):
    """Native doubles on the device (the reference keeps hi/lo f32 pairs and
    allows 2^-40 relative error; here the values come back bit for bit)."""
    wg, dev = cls
    data = np.array([1 / 3, np.pi, -2.5, 100.125])
    m = wg.GpuMatrix.from_(dev, data, 2, 2)
    assert m.dtype is np.float64
    back = m.read()
    m.destroy()
    assert back.tobytes() == data.tobytes()


def test_matrix_from_rejects_bad_arguments(cls):
    wg, dev = cls
    f = wg.GpuMatrix.from_
    with pytest.raises(wg.Error, match="Float32Array, Float64Array, Complex32Array, or Complex64Array"):
        f(dev, [1, 2, 3, 4], 2, 2)
    with pytest.raises(wg.Error, match="lda must be an integer >= cols"):
        f(dev, np.zeros(4, np.float32), 2, 2, 1)
    with pytest.raises(wg.Error, match="lda must be an integer >= rows"):
        f(dev, np.zeros(4, np.float32), 2, 2, 1, "column-major")
    with pytest.raises(wg.Error, match="data does not have enough elements"):
        f(dev, np.zeros(5, np.float32), 2, 2, 3)
    with pytest.raises(wg.Error, match="layout must be 'row-major' or 'column-major'"):
        f(dev, np.zeros(4, np.float32), 2, 2, None, "bogus")
    with pytest.raises(wg.Error, match="rows must be a positive integer"):
        f(dev, np.zeros(4, np.float32), 0, 2)
    with pytest.raises(wg.Error, match="cols must be a positive integer"):
        f(dev, np.zeros(4, np.float32), 2, 0)
    with pytest.raises(wg.Error, match="rows must be a positive integer"):
        f(dev, np.zeros(4, np.float32), 1.5, 2)
    with pytest.raises(wg.Error, match="lda must be an integer"):
        f(dev, np.zeros(8, np.float32), 2, 2, 2.5)


def test_matrix_default_lda_is_rows_for_column_major(cls):
    wg, dev = cls
    m = wg.GpuMatrix.from_(dev, np.array([1, 2, 3, 4], np.float32), 2, 2, None, "column-major")
    assert m.lda == 2
    back = m.read()
    m.destroy()
    assert back.tolist() == [1, 2, 3, 4]


def test_matrix_and_vector_without_device_use_get_device(rt):
    wg, _ = rt
    dev = wg.init()
    m = wg.GpuMatrix(object(), 1, 1, 1)
    assert m.device is wg.getDevice() is dev
    m2 = wg.GpuMatrix.from_(np.array([1, 2, 3, 4], np.float32), 2, 2)
    assert m2.device is dev
    m2.destroy()
    v = wg.GpuVector.from_(np.array([1, 2, 3], np.float64))
    assert v.device is dev and v.read().tolist() == [1, 2, 3]
    v.destroy()


def test_vector_round_trip_and_reject(cls):
    wg, dev = cls
    v = wg.GpuVector.from_(dev, np.array([1.5, -2, 3], np.float32))
    assert v.read().tolist() == [1.5, -2, 3]
    v.destroy()
    with pytest.raises(wg.Error, match="Float32Array, Float64Array"):
        wg.GpuVector.from_(dev, [1, 2, 3])


def test_read_after_destroy_is_refused(cls):
    wg, dev = cls
    m = wg.GpuMatrix.from_(dev, np.ones(4, np.float32), 2, 2)
    m.destroy()
    with pytest.raises(wg.Error, match="destroyed"):
        m.read()


# ---- examples/init-two-gpus/init-two-gpus.js on two GPUs ---------------------

@pytest.mark.gpu
def test_two_devices_run_concurrently(wg, oracle):
    """Two handles on two GPUs (high-performance -> first ordinal, low-power -> last),
    an sgemm on each from two threads at once, both checked against the oracle."""
    if wg._native.device_count() < 2:
        pytest.skip("needs two GPUs")
    d_gpu = wg.init(powerPreference="high-performance", device=None)
    i_gpu = wg.init(powerPreference="low-power", device=None)
    assert d_gpu.ordinal != i_gpu.ordinal
    n, k = 1024, 512
    res, errs = {}, []

    def run(dev, seed):
        try:
            A = wg.randomFloat32Array(n * k, -1, 1, seed)
            B = wg.randomFloat32Array(k * n, -1, 1, seed + 1)
            C = wg.randomFloat32Array(n * n, -1, 1, seed + 2)
            out = wg.sgemm(dev, "no-transpose", "no-transpose", n, n, k, 1.5, A, n, B, k, 0.5, C, n,
                           "column-major")["C"]
            res[seed] = (A, B, C, out)
        except Exception as e:  # noqa: BLE001 (reported below)
            errs.append(e)

    threads = [threading.Thread(target=run, args=(d, s)) for d, s in ((d_gpu, 10), (i_gpu, 20))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errs, errs
    for seed, (A, B, C, out) in res.items():
        truth, absab = oracle.sgemm_truth(0, 0, n, n, k, 1.5, A, n, B, k, 0.5, C, n)
        bound = oracle.sgemm_bound(n, n, k, 1.5, absab, 0.5, C, n)
        assert np.all(np.abs(oracle.block(out, n, n, n).astype(np.float64) - oracle.dense(truth, n, n)) <= bound)
    wg.cleanup(i_gpu)
    wg.cleanup(d_gpu)
