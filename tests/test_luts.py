"""The committed device LUT header equals the reference's ROM images and is
what gen_luts.py produces."""
import os
import re

import numpy as np

from fable5_llm_b200 import gen_luts

HDR = os.path.join(os.path.dirname(gen_luts.__file__), "csrc", "f5_luts.h")


def parse_header():
    out = {}
    for name, body in re.findall(r"#define F5_LUT_(\w+)_INIT \{([^}]*)\}", open(HDR).read()):
        out[name] = np.array([int(v) for v in body.split(",")], dtype=np.int64)
    return out


def test_header_is_generated():
    assert open(HDR).read() == gen_luts.render()


def test_header_matches_reference_roms(golden):
    r = golden("roms")
    h = parse_header()
    for name in ("rsqrt", "recip", "exp2", "sigmoid", "softplus"):
        assert np.array_equal(h[name.upper()], r[name]), name
