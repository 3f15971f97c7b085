"""Build the Linux LD_PRELOAD socket shaper: ``python infra/build_socket_shaper.py [--output PATH]``."""

from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
from pathlib import Path

PROJECT_ROOT = Path(__file__).resolve().parents[1]
SOURCE_PATH = PROJECT_ROOT / "infra" / "socket_shaper.c"
OUTPUT_PATH = PROJECT_ROOT / "infra" / "socket_shaper.so"


def build_socket_shaper(source: Path = SOURCE_PATH, output: Path = OUTPUT_PATH, force: bool = False) -> Path:
    """Compile ``source`` into ``output`` unless the shared object is already newer than the source."""
    if sys.platform != "linux":
        raise RuntimeError("socket shaper is only supported on Linux")
    if not force and output.exists() and output.stat().st_mtime >= source.stat().st_mtime:
        return output
    cc = shutil.which("cc") or shutil.which("gcc")
    if cc is None:
        raise FileNotFoundError("missing C compiler: expected 'cc' or 'gcc'")
    output.parent.mkdir(parents=True, exist_ok=True)
    subprocess.run([cc, "-O2", "-Wall", "-shared", "-fPIC", "-o", str(output), str(source), "-ldl", "-pthread", "-lrt"],
                   check=True, cwd=PROJECT_ROOT)
    return output


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--output", type=str, default=str(OUTPUT_PATH))
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build_socket_shaper(SOURCE_PATH, Path(args.output), force=args.force))


if __name__ == "__main__":
    main()
