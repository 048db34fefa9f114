"""Write ``reference_fixtures.json``: the reduce/scan known-answer cases that the
hephaestus test suites pin, transcribed from their sources.

Each case records the reference file:line it comes from (paths inside the
hephaestus project), its operands and the expected output (or the expected
error).  Literal expectations are copied from the reference's assertions;
where the reference computes its expectation with a loop over a generated
input (crates/hephaestus-cuda/tests/contract.rs), the same loop is restated
here in exact Python integer arithmetic, independent of the oracle under test.

Run: ``python tests/golden/make_reference_fixtures.py`` (no GPU, no reference
checkout needed).
"""
from __future__ import annotations

import json
import math
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))
CONF = "crates/hephaestus-conformance/src"
CONTRACT = "crates/hephaestus-cuda/tests/contract.rs"

F32_MAX = struct.unpack("<f", struct.pack("<f", 3.402823466e38))[0]


def f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


def cc(shape):
    strides, acc = [], 1
    for extent in reversed(shape):
        strides.insert(0, acc)
        acc *= max(extent, 1)
    return {"shape": list(shape), "strides": strides, "offset": 0}


def lay(shape, strides, offset=0):
    return {"shape": list(shape), "strides": list(strides), "offset": offset}


cases = []


def add(**kw):
    cases.append(kw)


# ---------------------------------------------------------------- full reduction
FULL_FIX = [1.0, 2.0, 3.0, 2.0] * 3  # conformance full_reduction.rs:58-60
for op, exp, line in [("sum", 24.0, 112), ("prod", 1728.0, 117), ("min", 1.0, 122),
                      ("max", 3.0, 127)]:
    add(id=f"conf_full_{op}", source=f"{CONF}/full_reduction.rs:{line}", kind="reduce_full",
        dtype="f32", input=FULL_FIX, layout=cc([3, 4]), op=op, expected=[exp])
for op, exp, line in [("sum", 24.0, 136), ("prod", 1728.0, 141)]:
    add(id=f"conf_full_transposed_{op}", source=f"{CONF}/full_reduction.rs:{line}",
        kind="reduce_full", dtype="f32", input=FULL_FIX, layout=lay([4, 3], [1, 4]), op=op,
        expected=[exp])
add(id="conf_full_diagonal_trace", source=f"{CONF}/full_reduction.rs:152-171", kind="reduce_full",
    dtype="f32", input=[float(v) for v in range(1, 10)], layout=lay([3], [4]), op="sum",
    expected=[15.0])
add(id="conf_full_prepared_rebind", source=f"{CONF}/full_reduction.rs:176-208",
    kind="reduce_full_prepared", dtype="f32", input=FULL_FIX, layout=cc([3, 4]), op="prod",
    rewrite=[2.0] * 12, expected=[1728.0], expected_after_rewrite=[4096.0])
add(id="conf_full_rejects_two_element_output", source=f"{CONF}/full_reduction.rs:214-231",
    kind="reduce_full", dtype="f32", input=FULL_FIX, layout=cc([3, 4]), op="sum",
    out_layout=cc([2]), out_init=[9.0, 9.0],
    error="full reduction output must have exactly 1 element")

# contract.rs:575-622 — sums at sizes {0,1,255,256,257,1027}
for n in [0, 1, 255, 256, 257, 1027]:
    fvals = [i * 0.5 for i in range(n)]
    add(id=f"contract_sum_f32_{n}", source=f"{CONTRACT}:575-622", kind="reduce_full",
        dtype="f32", input=fvals, layout=cc([n]), op="sum", expected=[sum(fvals)])
    uvals = list(range(n))
    add(id=f"contract_sum_u32_{n}", source=f"{CONTRACT}:575-622", kind="reduce_full",
        dtype="u32", input=uvals, layout=cc([n]), op="sum", expected=[sum(uvals) % 2**32])
    ivals = [i if i % 2 == 0 else -i for i in range(n)]
    add(id=f"contract_sum_i32_{n}", source=f"{CONTRACT}:575-622", kind="reduce_full",
        dtype="i32", input=ivals, layout=cc([n]), op="sum", expected=[sum(ivals)])
    # contract.rs:625-667 — f32 min/max of sin(i*12.34-100); empty -> +/-f32::MAX
    svals = [f32(math.sin(f32(f32(i * f32(12.34)) - 100.0))) for i in range(n)]
    add(id=f"contract_min_f32_{n}", source=f"{CONTRACT}:625-667", kind="reduce_full",
        dtype="f32", input=svals, layout=cc([n]), op="min",
        expected=[min(svals) if n else F32_MAX])
    add(id=f"contract_max_f32_{n}", source=f"{CONTRACT}:625-667", kind="reduce_full",
        dtype="f32", input=svals, layout=cc([n]), op="max",
        expected=[max(svals) if n else -F32_MAX])

# contract.rs:693-735 — u32 (i % 17) over 1027, and the empty sum
mod17 = [i % 17 for i in range(1027)]
for op, exp in [("sum", sum(mod17)), ("min", 0), ("max", 16)]:
    add(id=f"contract_prepared_u32_{op}", source=f"{CONTRACT}:693-735", kind="reduce_full",
        dtype="u32", input=mod17, layout=cc([1027]), op=op, expected=[exp])
add(id="contract_prepared_u32_empty_sum", source=f"{CONTRACT}:730-735", kind="reduce_full",
    dtype="u32", input=[], layout=cc([0]), op="sum", expected=[0])

# ---------------------------------------------------------------- axis reduction
AXIS_FIX = [float(v) for v in range(1, 13)]  # conformance axis_reduction.rs:59-61
add(id="conf_axis_prod_axis0", source=f"{CONF}/axis_reduction.rs:130", kind="reduce_axis",
    dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=0, op="prod",
    expected=[45.0, 120.0, 231.0, 384.0])
add(id="conf_axis_prod_axis1", source=f"{CONF}/axis_reduction.rs:149", kind="reduce_axis",
    dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=1, op="prod",
    expected=[24.0, 1680.0, 11880.0])
add(id="conf_axis_prod_transposed", source=f"{CONF}/axis_reduction.rs:159-200",
    kind="reduce_axis", dtype="f32", input=AXIS_FIX, layout=lay([4, 3], [1, 4]), axis=1,
    op="prod", expected=[45.0, 120.0, 231.0, 384.0])
add(id="conf_axis_rejects_axis2", source=f"{CONF}/axis_reduction.rs:204-237", kind="reduce_axis",
    dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=2, op="prod", out_layout=cc([1, 4]),
    out_init=[9.0] * 4, error="axis 2 is out of bounds for rank-2 reduction")
add(id="conf_axis_prepared_rebind", source=f"{CONF}/axis_reduction.rs:241-307",
    kind="reduce_axis_prepared", dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=0,
    op="prod", rewrite=[2.0] * 12, expected=[45.0, 120.0, 231.0, 384.0],
    expected_after_rewrite=[8.0, 8.0, 8.0, 8.0])
add(id="conf_axis_sum_axis0", source=f"{CONF}/axis_reduction.rs:311-382", kind="reduce_axis",
    dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=0, op="sum",
    expected=[15.0, 18.0, 21.0, 24.0])
add(id="conf_axis_rejects_wrong_output", source=f"{CONF}/axis_reduction.rs:385-419",
    kind="reduce_axis", dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=0, op="prod",
    out_layout=cc([1, 3]), out_init=[9.0] * 3,
    error_prefix="axis reduction output shape mismatch")
for op, axis, exp, line in [("min", 0, [1.0, 2.0, 3.0, 4.0], 456),
                            ("max", 0, [9.0, 10.0, 11.0, 12.0], 468),
                            ("min", 1, [1.0, 5.0, 9.0], 483),
                            ("max", 1, [4.0, 8.0, 12.0], 495),
                            ("mean", 0, [5.0, 6.0, 7.0, 8.0], 535),
                            ("mean", 1, [2.5, 6.5, 10.5], 551)]:
    add(id=f"conf_axis_{op}_axis{axis}", source=f"{CONF}/axis_reduction.rs:{line}",
        kind="reduce_axis", dtype="f32", input=AXIS_FIX, layout=cc([3, 4]), axis=axis, op=op,
        expected=exp)

C6 = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]  # contract.rs:1420
add(id="contract_axis_sum_axis0", source=f"{CONTRACT}:1425-1437", kind="reduce_axis",
    dtype="f32", input=C6, layout=cc([2, 3]), axis=0, op="sum", expected=[5.0, 7.0, 9.0])
add(id="contract_axis_prod_axis0", source=f"{CONTRACT}:1439-1452", kind="reduce_axis",
    dtype="f32", input=C6, layout=cc([2, 3]), axis=0, op="prod", expected=[4.0, 10.0, 18.0])
add(id="contract_axis_prod_axis1", source=f"{CONTRACT}:1454-1466", kind="reduce_axis",
    dtype="f32", input=C6, layout=cc([2, 3]), axis=1, op="prod", expected=[6.0, 120.0])
add(id="contract_axis_prod_transposed", source=f"{CONTRACT}:1489-1503", kind="reduce_axis",
    dtype="f32", input=C6, layout=lay([3, 2], [1, 3]), axis=1, op="prod",
    expected=[4.0, 10.0, 18.0])
add(id="contract_axis_prod_empty", source=f"{CONTRACT}:1525-1540", kind="reduce_axis",
    dtype="f32", input=[], layout=cc([0, 2]), axis=0, op="prod", expected=[1.0, 1.0])
add(id="contract_axis_sum_empty_axis", source=f"{CONTRACT}:1636-1655", kind="reduce_axis",
    dtype="f32", input=[], layout=cc([3, 0]), axis=1, op="sum", out_init=[7.0] * 3,
    expected=[0.0, 0.0, 0.0])
add(id="contract_axis_prod_empty_axis", source=f"{CONTRACT}:1657-1671", kind="reduce_axis",
    dtype="f32", input=[], layout=cc([3, 0]), axis=1, op="prod", expected=[1.0, 1.0, 1.0])
add(id="contract_axis_min_empty_axis", source=f"{CONTRACT}:1673-1691", kind="reduce_axis",
    dtype="f32", input=[], layout=cc([3, 0]), axis=1, op="min", out_init=[7.0] * 3,
    error="min_axis is undefined for empty axis 1")

# ---------------------------------------------------------------------- scans
SCAN_FIX = [1.0, 2.0, 3.0, 2.0] * 3  # conformance scan.rs:46-48
for op, axis, rev, exp, line in [
    ("sum", 1, False, [1.0, 3.0, 6.0, 8.0] * 3, 98),
    ("sum", 1, True, [8.0, 7.0, 5.0, 2.0] * 3, 105),
    ("prod", 1, False, [1.0, 2.0, 6.0, 12.0] * 3, 113),
    ("sum", 0, False, [1.0, 2.0, 3.0, 2.0, 2.0, 4.0, 6.0, 4.0, 3.0, 6.0, 9.0, 6.0], 123),
]:
    add(id=f"conf_scan_{op}_axis{axis}_{'rev' if rev else 'fwd'}",
        source=f"{CONF}/scan.rs:{line}", kind="scan", dtype="f32", input=SCAN_FIX,
        layout=cc([3, 4]), axis=axis, op=op, reverse=rev, expected=exp)
add(id="conf_scan_rejects_axis2", source=f"{CONF}/scan.rs:128-150", kind="scan", dtype="f32",
    input=SCAN_FIX, layout=cc([3, 4]), axis=2, op="sum", reverse=False, out_init=[9.0] * 12,
    error="scan axis 2 is out of bounds for rank-2 scan")
add(id="conf_scan_prepared_rebind", source=f"{CONF}/scan.rs:155-205", kind="scan_prepared",
    dtype="f32", input=SCAN_FIX, layout=cc([3, 4]), axis=1, op="sum", reverse=False,
    rewrite=[1.0] * 12, expected=[1.0, 3.0, 6.0, 8.0] * 3,
    expected_after_rewrite=[1.0, 2.0, 3.0, 4.0] * 3)
add(id="contract_scan_2x2", source=f"{CONTRACT}:1729-1750", kind="scan", dtype="f32",
    input=[1.0, 2.0, 3.0, 4.0], layout=cc([2, 2]), axis=1, op="sum", reverse=False,
    expected=[1.0, 3.0, 3.0, 7.0])
add(id="contract_scan_suffix_sum_i32", source=f"{CONTRACT}:1755-1804", kind="scan", dtype="i32",
    input=[1, 2, 3, 4, 5, 6], layout=cc([2, 3]), axis=1, op="sum", reverse=True,
    expected=[6, 5, 3, 15, 11, 6])
P6 = [1, 2, 3, 4, 5, 6]
T23 = lay([2, 3], [1, 2])  # contract.rs:1814
add(id="contract_cumprod_transposed_axis1", source=f"{CONTRACT}:1807-1834", kind="scan",
    dtype="i32", input=P6, layout=T23, out_layout=cc([2, 3]), axis=1, op="prod", reverse=False,
    expected=[1, 3, 15, 2, 8, 48])
add(id="contract_cumprod_transposed_axis0", source=f"{CONTRACT}:1835-1848", kind="scan",
    dtype="i32", input=P6, layout=T23, out_layout=cc([2, 3]), axis=0, op="prod", reverse=False,
    expected=[1, 3, 5, 2, 12, 30])
add(id="contract_suffix_prod_transposed_axis1", source=f"{CONTRACT}:1849-1862", kind="scan",
    dtype="i32", input=P6, layout=T23, out_layout=cc([2, 3]), axis=1, op="prod", reverse=True,
    expected=[15, 15, 5, 48, 24, 6])
add(id="contract_suffix_prod_transposed_axis0", source=f"{CONTRACT}:1863-1881", kind="scan",
    dtype="i32", input=P6, layout=T23, out_layout=cc([2, 3]), axis=0, op="prod", reverse=True,
    expected=[2, 12, 30, 2, 4, 6])
add(id="contract_cumprod_empty", source=f"{CONTRACT}:1882-1895", kind="scan", dtype="i32",
    input=[], layout=cc([2, 0]), axis=1, op="prod", reverse=False, expected=[])
add(id="contract_cumprod_layout_rejected", source=f"{CONTRACT}:1896-1911", kind="scan",
    dtype="i32", input=P6, layout=lay([2, 3], [1, 2], 1), out_layout=cc([2, 3]), axis=1,
    op="prod", reverse=False, error_prefix="layout rejected:")
cols = 513
long_in = [i - 300 for i in range(2 * cols)]
long_exp = []
for r in range(2):
    acc = 0
    for v in long_in[r * cols:(r + 1) * cols]:
        acc += v
        long_exp.append(acc)
add(id="contract_scan_long_line_i32", source=f"{CONTRACT}:1913-1949", kind="scan", dtype="i32",
    input=long_in, layout=cc([2, cols]), axis=1, op="sum", reverse=False, expected=long_exp)

# ------------------------------------------------------- map reductions
MAPS = {"dot": 0, "trace": 1, "norm_l1": 2, "norm_l2": 3, "norm_max": 4}
add(id="contract_dot", source=f"{CONTRACT}:895-927", kind="map", map="dot", dtype="f32",
    input=[1.0, 2.0, 3.0, 4.0], layout=cc([4]), input_b=[5.0, 6.0, 7.0, 8.0], layout_b=cc([4]),
    expected=[70.0])
add(id="contract_trace", source=f"{CONTRACT}:929-953", kind="map", map="trace", dtype="f32",
    input=[float(v) for v in range(1, 10)], layout=lay([3], [4]), expected=[15.0])
add(id="contract_prepared_dot_rebind", source=f"{CONTRACT}:955-985", kind="map", map="dot", dtype="f32",
    input=[2.0, 2.0, 2.0, 2.0], layout=cc([4]), input_b=[5.0, 6.0, 7.0, 8.0], layout_b=cc([4]),
    expected=[52.0])
add(id="contract_prepared_dot_reversed", source=f"{CONTRACT}:988-1003", kind="map", map="dot", dtype="f32",
    input=[2.0, 2.0, 2.0, 2.0], layout=lay([4], [-1], 3), input_b=[5.0, 6.0, 7.0, 8.0], layout_b=cc([4]),
    expected=[52.0])
add(id="contract_norm_l2_transposed", source=f"{CONTRACT}:1005-1022", kind="map", map="norm_l2", dtype="f32",
    input=[1.0, 2.0, 3.0, 4.0], layout=lay([2, 2], [1, 2]), expected=[math.sqrt(30.0)],
    tolerance=2 * 1.1920929e-07 * math.sqrt(30.0))
add(id="contract_norm_l2_rewrite", source=f"{CONTRACT}:1023-1029", kind="map", map="norm_l2", dtype="f32",
    input=[4.0] * 4, layout=lay([2, 2], [1, 2]), expected=[8.0])
add(id="contract_empty_dot", source=f"{CONTRACT}:1034-1048", kind="map", map="dot", dtype="f32", input=[],
    layout=cc([0]), input_b=[], layout_b=cc([0]), expected=[0.0])
add(id="contract_empty_norm_l2", source=f"{CONTRACT}:1050-1060", kind="map", map="norm_l2", dtype="f32",
    input=[], layout=cc([0]), expected=[0.0])
add(id="contract_dot_shape_mismatch", source=f"{CONTRACT}:1062-1077", kind="map", map="dot", dtype="f32",
    input=[1.0, 2.0, 3.0, 4.0], layout=cc([4]), input_b=[5.0, 6.0, 7.0, 8.0], layout_b=cc([3]),
    error_prefix="dot product shape mismatch:")
add(id="contract_norm_layout_rejected", source=f"{CONTRACT}:1079-1090", kind="map", map="norm_l2", dtype="f32",
    input=[1.0, 2.0, 3.0, 4.0], layout=lay([3], [1], 2), error_prefix="layout rejected:")
for m, exp, line in [("norm_l1", 10.0, "1094-1111"), ("norm_l2", math.sqrt(30.0), "1112-1118"),
                     ("norm_max", 4.0, "1119-1124")]:
    add(id=f"contract_{m}", source=f"{CONTRACT}:{line}", kind="map", map=m, dtype="f32",
        input=[-1.0, 2.0, -3.0, 4.0], layout=cc([4]), expected=[exp],
        **({"tolerance": 1e-5} if m == "norm_l2" else {}))
add(id="contract_dot_reversed_values", source=f"{CONTRACT}:1128-1154", kind="map", map="dot", dtype="f32",
    input=[-1.0, 2.0, -3.0, 4.0], layout=lay([4], [-1], 3), input_b=[1.0, 2.0, 3.0, 4.0], layout_b=cc([4]),
    expected=[0.0])
add(id="contract_norm_l1_reversed", source=f"{CONTRACT}:1155-1156", kind="map", map="norm_l1", dtype="f32",
    input=[-1.0, 2.0, -3.0, 4.0], layout=lay([4], [-1], 3), expected=[10.0])

# ---------------------------------------------------------------- widths
add(id="contract_width_192", source=f"{CONTRACT}:670-690", kind="width", width=192,
    error="reduction block width 192 must be a power of two")
add(id="contract_width_3", source=f"{CONTRACT}:1711-1725", kind="width", width=3,
    error="reduction block width 3 must be a power of two")
add(id="core_pass_count", source="crates/hephaestus-core/src/domain/reduction.rs:356-366",
    kind="pass_count", cases=[[0, 256, 0], [1, 256, 0], [256, 256, 1], [257, 256, 2],
                              [1 << 20, 256, 3], [1027, 128, 2]])

if __name__ == "__main__":
    path = os.path.join(HERE, "reference_fixtures.json")
    with open(path, "w") as fh:
        json.dump({"generator": "tests/golden/make_reference_fixtures.py", "cases": cases}, fh,
                  indent=1)
    print(f"wrote {len(cases)} cases to {path}")
