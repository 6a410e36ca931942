"""The B200 GPU profile for kdev's floor tools (schema kdev.gpu/1).

kdev ships only an H200 profile (src/kdev/data/gpus/h200.toml) and looks for others under
$KDEV_HOME/gpus/<name>.toml (src/kdev/floor/gpus.py:139-160), so `install_profile()` copies this
package's b200.toml there.  `profile_dict()` returns the parsed profile without kdev.
"""
from __future__ import annotations

import os
import shutil
import tomllib
from pathlib import Path

PROFILE = Path(__file__).resolve().parent / "b200.toml"


def profile_dict() -> dict:
    """The parsed b200 profile."""
    return tomllib.loads(PROFILE.read_text(encoding="utf-8"))


def install_profile(home: str | None = None, overwrite: bool = False) -> Path:
    """Copies b200.toml to <home or $KDEV_HOME>/gpus/b200.toml and returns that path.  An existing file
    (a user's measured overrides) is kept unless overwrite=True."""
    h = home or os.environ.get("KDEV_HOME")
    if not h:
        raise ValueError("no kdev home: pass home= or set KDEV_HOME")
    dst = Path(h).expanduser() / "gpus" / "b200.toml"
    dst.parent.mkdir(parents=True, exist_ok=True)
    if overwrite or not dst.exists():
        shutil.copyfile(PROFILE, dst)
    return dst
