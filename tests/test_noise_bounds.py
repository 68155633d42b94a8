"""The FP32 noise bounds the certified draws rely on hold for every one of
the 2^32 Philox words (run on the GPU; about a second)."""
import json
import subprocess

import pytest

from tests import noise_bounds

pytestmark = pytest.mark.gpu


def test_noise_bounds_hold_for_every_word():
    binary = noise_bounds.build()
    result = subprocess.run([str(binary)], capture_output=True, text=True, timeout=600)
    report = json.loads(result.stdout.strip().splitlines()[-1])
    print(report)
    assert result.returncode == 0 and report["passed"], report
    assert report["error_violations"] == 0 and report["screen_violations"] == 0
