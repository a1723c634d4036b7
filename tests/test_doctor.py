"""The environment report runs anywhere and says what is missing."""
import json
import subprocess
import sys


def test_doctor_reports_json():
    out = subprocess.run([sys.executable, "-m", "weightbridge_b200.doctor"], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    rep = json.loads(out.stdout)
    assert rep["extension"]["loaded"] is True
    assert isinstance(rep["gpus"], list) and isinstance(rep["notes"], list)
