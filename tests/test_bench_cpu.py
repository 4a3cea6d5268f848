"""bench.py's CPU baselines on the CPU: the reference's own code (oracle/_ref)
timed on short samples returns positive rates in the units of the GPU numbers
they sit beside, and each lands beside its configuration's extra."""
import pytest

import bench
import oracle

pytestmark = pytest.mark.skipif(oracle.ref() is None, reason="oracle/_ref (reference build) not present")


def test_reference_samples_have_the_gpu_units():
    ref = bench.RefConfigs(min_seconds=0.02)
    c1 = ref.config1()
    assert c1["unit"] == "GB/s" and c1["value"] > 0 and c1["kind"] == "reference" and c1["cores"] >= 1
    c3 = ref.config3()
    assert c3["prefill"]["unit"] == "tok/s" and c3["decode"]["unit"] == "GB/s"
    assert c3["prefill"]["cores"] == 1  # the reference's token loop is serial
    # configs 4 and 5 run the same two samplers at full size (seconds of cache
    # fills); here the samplers alone, on small caches, windowed and not
    k, v = ref._rows(1, 1, 300, 4 * 256), ref._rows(1, 2, 300, 4 * 256)
    q = ref._rows(1, 3, 300, 8 * 256)
    for window in (0, 64):
        assert ref.prefill_seconds(k, v, q, 4, 256, 8, None, window, 268, 32) > 0
        assert ref.decode_seconds(k, v, q[-1:].copy(), 4, 256, 8, None, window) > 0


def test_baselines_attach_beside_each_extra():
    extra = {"config1": {"value": 1.0}, "config3": {"prefill_chunk64": {}, "decode": {}},
             "config4": {"prefill": {}, "decode": {}}, "config5": {"error": "not run"}}

    class Stub(bench.RefConfigs):
        def __init__(self):
            self.cores, self.kind = 1, "reference"

        def config1(self):
            return self.line(1.0, "GB/s", "c1")

        def config3(self):
            return {"prefill": self.line(2.0, "tok/s", "c3"), "decode": self.line(3.0, "GB/s", "c3")}

        def config4(self):
            return {"prefill": self.line(4.0, "TFLOP/s", "c4"), "decode": self.line(5.0, "GB/s", "c4")}

        def config5(self):
            raise AssertionError("an extra that failed gets no baseline")

    real = bench.RefConfigs
    bench.RefConfigs = Stub
    try:
        bench.cpu_baselines(extra)
    finally:
        bench.RefConfigs = real
    assert extra["config1"]["cpu_baseline"]["value"] == 1.0
    assert extra["config3"]["prefill_chunk64"]["cpu_baseline"]["unit"] == "tok/s"
    assert extra["config3"]["decode"]["cpu_baseline"]["value"] == 3.0
    assert extra["config4"]["prefill"]["cpu_baseline"]["unit"] == "TFLOP/s"
    assert "cpu_baseline" not in extra["config5"]
