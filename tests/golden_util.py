"""Helpers shared by the tests that read tests/golden/reference_fixtures.json."""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
DT = {"f32": np.float32, "f64": np.float64, "u32": np.uint32, "i32": np.int32, "i64": np.int64}
OPS = {"sum": 0, "prod": 1, "min": 2, "max": 3, "mean": 4}


def load_cases():
    with open(os.path.join(HERE, "golden", "reference_fixtures.json")) as fh:
        return json.load(fh)["cases"]


def cases_of_kind(*kinds):
    return [c["id"] for c in load_cases() if c["kind"] in kinds]


def input_array(c):
    return np.array(c["input"], dtype=DT[c["dtype"]])
