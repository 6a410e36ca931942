"""The B200 GPU profile (kdb200/gpus/b200.toml) read by kdev's own profile loader and roofline
(src/kdev/floor/gpus.py, src/kdev/floor/roofline.py), CPU only.  Skipped when kdev's sources are absent."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

from kdb200 import gpus

# kdev itself: $KDEV_SRC (a source tree's `src`), else its offline install under baseline/_ref
KDEV_SRC = Path(os.environ["KDEV_SRC"]) if os.environ.get("KDEV_SRC") else Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def test_profile_parses_without_kdev():
    d = gpus.profile_dict()
    assert d["schema"] == "kdev.gpu/1" and d["name"] == "b200" and d["sm_count"] == 148
    assert d["flush_bytes"] >= 4 * d["l2_bytes"]
    for k, v in d["measured"].items():
        assert v["value"] > 0 and v["unit"] and v["source"], k


def test_install_keeps_user_overrides(tmp_path):
    dst = gpus.install_profile(str(tmp_path))
    assert dst == tmp_path / "gpus" / "b200.toml" and dst.read_text() == gpus.PROFILE.read_text()
    dst.write_text(dst.read_text().replace("sm_count = 148", "sm_count = 148  # edited"))
    gpus.install_profile(str(tmp_path))
    assert "# edited" in dst.read_text()
    gpus.install_profile(str(tmp_path), overwrite=True)
    assert "# edited" not in dst.read_text()


@pytest.mark.skipif(not (KDEV_SRC / "kdev" / "floor" / "gpus.py").exists(), reason="kdev sources not available")
def test_kdev_loads_profile_and_floors_the_projection(tmp_path):
    sys.path.insert(0, str(KDEV_SRC))
    try:
        from kdev.floor import gpus as kg
        from kdev.floor import roofline as kr
    finally:
        sys.path.remove(str(KDEV_SRC))
    gpus.install_profile(str(tmp_path))
    prof = kg.load_profile("b200", home=str(tmp_path))
    assert prof.sm_count == 148 and prof.l2_bytes == 132120576 and prof.peak["bf16_tflops"] == 2250
    assert prof.const("stream_tbps") == pytest.approx(6.5485)
    assert kg.detect_name("NVIDIA B200") == "b200"
    # 4096 x 7168 x 7168 projection: compute bound, 187 us at the datasheet peak
    m, n, k = 4096, 7168, 7168
    f = kr.roofline(prof, 2.0 * (m * k + n * k + m * n), 2.0 * m * n * k, "bf16")
    assert f.bound == "compute" and f.floor_us == pytest.approx(2.0 * m * n * k / 2250e12 * 1e6)
    # 16 x 7168 x 7168: memory bound
    f16 = kr.roofline(prof, 2.0 * (16 * k + n * k + 16 * n), 2.0 * 16 * n * k, "bf16")
    assert f16.bound == "memory" and f16.floor_us_achievable > f16.mem_us_peak
