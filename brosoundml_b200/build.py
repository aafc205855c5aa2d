"""Build step for libbsml_b200.so (nvcc, sm_100a)."""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-C", HERE, f"-j{jobs}"], check=True)
    return os.path.join(HERE, "libbsml_b200.so")


if __name__ == "__main__":
    print(build())
