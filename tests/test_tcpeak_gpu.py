"""The tensor-core throughput probe (sicu_tc_peak) that gives the prefill
roofline its measured kind::f16 and kind::i8 denominators: it runs both
kinds to completion (no bounded wait gives up), reports a time and a rate in
a plausible range, and the int8 kind retires more multiply-adds per second
than the f16 kind on the same SMs."""

from __future__ import annotations

import pytest

from siphon_b200.lib import TC_F16, TC_I8, SicuError

pytestmark = pytest.mark.gpu


def test_tc_peak_both_kinds(sicu):
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    f16_ms, f16 = sicu.tc_peak(TC_F16, 400, sms)
    i8_ms, i8 = sicu.tc_peak(TC_I8, 400, sms)
    assert f16_ms > 0 and i8_ms > 0
    assert 100.0 < f16 < 10000.0, f"kind::f16 {f16:.1f} TFLOP/s"
    assert 100.0 < i8 < 20000.0, f"kind::i8 {i8:.1f} TOP/s"
    assert i8 > f16, (i8, f16)
    assert sicu.status() == 0


def test_tc_peak_rejects_bad_arguments(sicu):
    with pytest.raises(SicuError):
        sicu.tc_peak(7, 10, 1)
    with pytest.raises(SicuError):
        sicu.tc_peak(TC_F16, 0, 1)
