#!/usr/bin/env python3
"""Emmy kernel IR -> sm_100a PTX (drop-in for the reference's CLI, compile.py:1802-1817).

    python compile.py path/to/kernel.ir.json > out.ptx
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from emmy_ptx_b200.compiler import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main(sys.argv))
