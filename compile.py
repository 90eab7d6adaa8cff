#!/usr/bin/env python3
"""Compile one Emmy Kernel IR to sm_100a PTX.

    python compile.py path/to/kernel.ir.json > out.ptx

Reads meta.json next to the IR for the parameter order.  The same invocation
contract as the reference's compile.py: exactly one argument (else usage on
stderr and exit 2), PTX only on stdout, a traceback and non-zero exit for IR
this back end does not support.
"""

from __future__ import annotations

import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "emmy-hackathon-2026_b200"))

from compiler import compile_kernel, load  # noqa: E402


def main() -> int:
    if len(sys.argv) != 2:
        print(__doc__, file=sys.stderr)
        return 2
    sys.stdout.write(compile_kernel(load(sys.argv[1])))
    return 0


if __name__ == "__main__":
    sys.exit(main())
