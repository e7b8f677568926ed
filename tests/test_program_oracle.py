"""The CPU program oracle (oracle/program_oracle.py) pinned against the
reference's own whole-program expectations: the add -> mm program of
tests/api/program.test.ts:54-68 (expected [112, 160, 240, 352]) and the
PyTorch output fixtures of tests/program/yolo26n.test.ts:69-94 (fp32,
every element within 0.01) and depthart.test.ts:60-101 (fp32, within 1.0),
with the fp16 programs checked by those tests' fp16 criteria."""
import json
import os

import numpy as np
import pytest

import program_oracle

ASSETS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "_assets")


def test_add_mm_program():
    prog = {
        "version": "1",
        "chain": [{"name": "aten.add.Tensor", "args": [0, 1, 2, 3]},
                  {"name": "aten.mm.default", "args": [3, 4, 5]}],
        "values": [
            {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 0},
            {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 1},
            {"type": "scalar", "value": 1.5},
            {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 2},
            {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 3},
            {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 0},
        ],
        "inputIds": [0, 1, 4], "outputIds": [5],
        "memoryPlan": {"pools": [{"id": i, "size": 16} for i in range(4)]},
    }
    a = np.array([1, 2, 3, 4], np.float32)
    b = np.array([10, 20, 30, 40], np.float32)
    (out,) = program_oracle.run_program(prog, b"", [a, b, a])
    np.testing.assert_array_equal(out.reshape(-1), [112, 160, 240, 352])


def fixture_case(model, fp16):
    d = os.path.join(ASSETS, model)
    path = os.path.join(d, "program-fp16.json" if fp16 else "program.json")
    if not os.path.exists(path):
        pytest.skip("model artefacts not present (run __graft_entry__.build())")
    prog = json.load(open(path))
    w = open(os.path.join(d, "weights-fp16.bin" if fp16 else "weights.bin"), "rb").read()
    n = int(np.prod(prog["values"][prog["inputIds"][0]]["shape"]))
    x = ((np.arange(n) % 251) / 250.0 - 0.5).astype(np.float16 if fp16 else np.float32)
    (y,) = program_oracle.run_program(prog, w, [x])
    ref = np.fromfile(os.path.join(d, "reference-output.f32"), dtype=np.float32)
    return y.reshape(-1).astype(np.float64), ref.astype(np.float64)


def test_yolo26n_fp32_matches_fixture():
    y, ref = fixture_case("yolo26n", False)
    assert np.abs(y - ref).max() <= 0.01


def test_yolo26n_fp16_matches_fixture():
    y, ref = fixture_case("yolo26n", True)
    assert np.mean(np.abs(y - ref) > 0.5) <= 0.05


def test_depthart_fp32_matches_fixture():
    y, ref = fixture_case("depthart", False)
    assert np.abs(y - ref).max() <= 1.0
