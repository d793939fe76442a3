"""CPU checks of the C ABI library: it builds, loads without a GPU, exports
every symbol include/wohper_b200.h declares, and the host-side pieces the
kernels depend on (act-quant exponent table, E4M3 rounding) match the
reference's semantics as restated by the oracle and measured from libm."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import oracle as O
import wohper_b200 as W

ROOT = Path(__file__).resolve().parents[1]


def test_library_loads_and_exports_header_symbols():
    L = W.lib()
    header = (ROOT / "include" / "wohper_b200.h").read_text()
    declared = set(re.findall(r"\b(wh_[a-z0-9_]+)\s*\(", header))
    declared -= {"wh_status"}
    assert declared, "no declarations parsed"
    missing = [name for name in sorted(declared) if not hasattr(L, name)]
    assert not missing, f"library lacks {missing}"
    assert set(W.EXPORTS) == declared
    assert L.wh_version() >= 100


def test_status_codes_mirror_reference_error_enum():
    header = (ROOT / "include" / "wohper_b200.h").read_text()
    # DeepSeekV4KernelError (src/deepseek_v4.rs:398-408) in declaration order
    order = ["EMPTY_SHAPE", "INVALID_SHAPE", "PACKED_WEIGHT_TOO_SMALL", "SCALE_TOO_SMALL",
             "INPUT_TOO_SMALL", "OUTPUT_TOO_SMALL", "SCRATCH_TOO_SMALL", "NON_FINITE_OUTPUT"]
    for i, name in enumerate(order, start=1):
        assert re.search(rf"WH_ERR_{name}\s*=\s*{i}\b", header), name
        assert getattr(O, f"ERR_{name}") == i


def test_fp4_scratch_len_matches_reference():
    assert W.lib().wh_fp4_expert_scratch_len(2048) == 4096 == O.lib().orc_fp4_expert_scratch_len(2048)


def _libm_ceil_log2f():
    m = C.CDLL("libm.so.6")
    m.log2f.argtypes = [C.c_float]
    m.log2f.restype = C.c_float
    return lambda q: float(np.ceil(np.float32(m.log2f(float(q)))))


def test_act_quant_exponent_table_matches_libm():
    table = np.zeros(256, np.uint32)
    W.lib().wh_debug_act_quant_table(table.ctypes.data_as(C.c_void_p))
    ceil_log2f = _libm_ceil_log2f()
    g = np.random.default_rng(7)
    # q = amax/448 with amax >= 1e-4 -> biased exponent >= 105
    for E in list(range(100, 160)) + [200, 254]:
        k = E - 127
        thr = int(table[E])
        ms = {0, 1, 2, 3, thr - 2, thr - 1, thr, thr + 1, thr + 2, (1 << 23) - 1}
        ms |= set(int(v) for v in g.integers(0, 1 << 23, size=40))
        for m in ms:
            if not 0 <= m < (1 << 23):
                continue
            q = np.array([(E << 23) | m], np.uint32).view(np.float32)[0]
            want = ceil_log2f(q)
            got = k if (m == 0 or m < thr) else k + 1
            assert want == got, (E, m, thr, want, got)


def test_act_quant_exponent_table_is_monotone_band():
    # The table encodes "ceil(log2f(q)) == k only in a band just above 2^k":
    # check every mantissa of that band and well past it for a few exponents,
    # so the binary search that built it cannot have hidden a non-monotone step.
    table = np.zeros(256, np.uint32)
    W.lib().wh_debug_act_quant_table(table.ctypes.data_as(C.c_void_p))
    ceil_log2f = _libm_ceil_log2f()
    for E in (110, 117, 120, 124, 127, 130):
        k = E - 127
        thr = int(table[E])
        for m in range(0, thr + 2048):
            q = np.array([(E << 23) | m], np.uint32).view(np.float32)[0]
            assert (ceil_log2f(q) == k) == (m == 0 or m < thr), (E, m, thr)


def test_e4m3_rounding_matches_oracle_ties_to_lower():
    lut = O.luts()["sorted"]
    grid = np.unique(lut[(lut >= -448) & (lut <= 448)])
    mids = (grid[:-1].astype(np.float64) + grid[1:]) / 2
    cand = [grid, mids.astype(np.float32)]
    for d in (1, 2, 3):
        cand.append(np.nextafter(mids.astype(np.float32), np.float32(np.inf)))
        cand.append(np.nextafter(mids.astype(np.float32), np.float32(-np.inf)))
    g = np.random.default_rng(11)
    cand.append(g.uniform(-448, 448, 200000).astype(np.float32))
    cand.append((g.uniform(-1, 1, 100000) * 0.02).astype(np.float32))
    cand.append(np.array([0.0, -0.0, 448.0, -448.0, 2.0**-10, -(2.0**-10), 1e-30, -1e-30],
                         np.float32))
    vals = np.concatenate(cand).astype(np.float32)
    got = np.zeros_like(vals)
    W.lib().wh_debug_e4m3_round_n(vals.ctypes.data_as(C.c_void_p),
                                  got.ctypes.data_as(C.c_void_p), vals.size)
    # oracle: blocks of 63 values plus an amax of 448 so the block scale is 1
    n = vals.size
    pad = (-n) % 63
    v = np.concatenate([vals, np.zeros(pad, np.float32)]).reshape(-1, 63)
    blocks = np.concatenate([np.full((v.shape[0], 1), 448.0, np.float32), v], axis=1)
    want = O.act_quant(blocks.reshape(-1), 64).reshape(-1, 64)[:, 1:].reshape(-1)[:n]
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
