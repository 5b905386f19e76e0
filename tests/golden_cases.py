"""Load the golden fixtures of tests/golden/ (outputs of the reference's own CUDA kernels,
written by tests/golden/make_golden.py) together with their regenerated inputs."""
import importlib.util
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)

SCAN_NAMES = list(make_golden.SCAN_CASES)
UPDATE_NAMES = list(make_golden.UPDATE_CASES)


def load(name):
    path = os.path.join(GOLDEN, name + ".npz")
    if not os.path.exists(path):
        raise FileNotFoundError(f"golden fixture {path} is missing; regenerate with tests/golden/make_golden.py")
    with np.load(path) as f:
        meta = json.loads(str(f["meta"]))
        arrays = {k: f[k] for k in f.files if k != "meta"}
    return meta, arrays


def scan_case(name):
    """(meta, arrays, inputs, length, dh_last, padding side); checks the input digest."""
    meta, arrays = load(name)
    case = tuple(make_golden.SCAN_CASES[name])
    assert tuple(meta["case"][:5]) == case[:5], f"{name}: fixture made for case {meta['case']}, test has {case}"
    inp, length, dh_last, digest = make_golden.scan_case_inputs(case)
    assert digest == meta["input_sha256"], f"{name}: regenerated inputs differ from the ones the fixture used"
    return meta, arrays, inp, length, dh_last, case[6]


def update_case(name):
    meta, arrays = load(name)
    case = tuple(make_golden.UPDATE_CASES[name])
    dec, digest = make_golden.update_case_inputs(case)
    assert digest == meta["input_sha256"], f"{name}: regenerated inputs differ from the ones the fixture used"
    return meta, arrays, dec
