"""Writes the golden fixtures of tests/golden/ from the reference itself.

    python tests/golden/make_golden.py

fp8_e4m3_reference.json: the 256 values of the reference's own
`fp8_e4m3_to_fp32` (hyperion_fa3_production_final.py:122-141), compiled for the
host from the reference's source by oracle/build.py into oracle/_ref/.  Values
are stored as float32 bit patterns (hex) so signed zeros and subnormals survive.

Needs the reference checkout (this container); the committed JSON is what the
tests read everywhere else.
"""
import ctypes
import json
import os
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import build as oracle_build  # noqa: E402


def main():
    so = oracle_build.build_ref(force=True)
    if so is None:
        raise SystemExit("reference checkout not found: set HYPERION_REFERENCE_DIR")
    ref = ctypes.CDLL(so)
    ref.ref_fp8_e4m3_to_fp32.restype = ctypes.c_float
    ref.ref_fp8_e4m3_to_fp32.argtypes = [ctypes.c_uint8]
    bits = ["%08x" % struct.unpack("<I", struct.pack("<f", ref.ref_fp8_e4m3_to_fp32(c)))[0] for c in range(256)]
    out = {
        "source": "hyperion_fa3_production_final.py:122-141 fp8_e4m3_to_fp32, compiled for the host",
        "generator": "tests/golden/make_golden.py",
        "f32_bits_hex": bits,
    }
    with open(os.path.join(HERE, "fp8_e4m3_reference.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", len(bits), "codes")


if __name__ == "__main__":
    main()
