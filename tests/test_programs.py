"""Program transforms (wgx.programs) on the reference's shipped models, on
the CPU: fp16 conversion pinned byte for byte against the shipped
program-fp16.json / weights-fp16.bin (made by
utils/convert_model_to_fp16.mjs), batch lift, spatial re-shape and seeded
random-init weights."""
import copy
import json
import os

import numpy as np
import pytest

from wgx import programs

ASSETS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "_assets")


def load(model, name):
    path = os.path.join(ASSETS, model, name)
    if not os.path.exists(path):
        pytest.skip("model artefacts not present (run __graft_entry__.build())")
    if name.endswith(".json"):
        return json.load(open(path))
    return open(path, "rb").read()


@pytest.mark.parametrize("model", ["yolo26n", "depthart", "selfie-segmentation"])
def test_fp16_conversion_matches_shipped(model):
    prog, w = load(model, "program.json"), load(model, "weights.bin")
    p16, w16 = programs.convert_to_fp16(prog, w, depthart_rebalance=(model == "depthart"))
    assert p16 == load(model, "program-fp16.json")
    assert w16 == load(model, "weights-fp16.bin")
    assert prog == load(model, "program.json")   # input untouched


def test_depthart_rebalance_checks_structure():
    prog, w = load("yolo26n", "program.json"), load("yolo26n", "weights.bin")
    with pytest.raises(ValueError, match="DepthART decoder changed"):
        programs.convert_to_fp16(prog, w, depthart_rebalance=True)


def test_batch_lift_yolo_shapes():
    prog = load("yolo26n", "program-fp16.json")
    lifted = programs.batch_lift(prog, 4)
    v = lifted["values"]
    assert v[lifted["inputIds"][0]]["shape"] == [4, 3, 640, 640]
    assert v[lifted["outputIds"][0]]["shape"] == [4, 84, 8400]
    bmm = [op for op in lifted["chain"] if op["name"] == "aten.bmm.default"]
    assert [v[a]["shape"] for a in bmm[0]["args"]] == [[8, 400, 32], [8, 32, 400], [8, 400, 400]]
    views = [op for op in lifted["chain"] if op["name"] == "aten.view_copy.default"]
    for op in views:
        items = v[op["args"][1]]["items"]
        out = v[op["args"][-1]]["shape"]
        assert items[0] == out[0] == 4 or items[0] == -1
    # constants are shared, not lifted
    for op in lifted["chain"]:
        if op["name"] == "et_vk.prepack.default":
            assert v[op["args"][0]]["shape"] == v[op["args"][1]]["shape"]
    # every pool holds its largest member
    sizes = {p["id"]: p["size"] for p in lifted["memoryPlan"]["pools"]}
    for t in v:
        if t["type"] == "tensor" and t.get("memObjId") is not None:
            assert sizes[t["memObjId"]] >= programs.tensor_bytes(t)
    assert programs.batch_lift(prog, 1) == prog


def test_batch_lift_rejects_mixing_images():
    prog = {
        "version": "1",
        "values": [
            {"type": "tensor", "shape": [1, 4], "dtype": "float32", "memObjId": 0},
            {"type": "tensor", "shape": [1, 4], "dtype": "float32", "memObjId": 1},
            {"type": "tensorlist", "items": [0, 1]},
            {"type": "scalar", "value": 0},
            {"type": "tensor", "shape": [2, 4], "dtype": "float32", "memObjId": 2},
        ],
        "chain": [{"name": "aten.cat.default", "args": [2, 3, 4]}],
        "inputIds": [0, 1], "outputIds": [4],
        "memoryPlan": {"pools": [{"id": i, "size": 32} for i in range(3)]},
    }
    with pytest.raises(ValueError, match="batch dimension"):
        programs.batch_lift(prog, 2)
    ok = copy.deepcopy(prog)
    ok["values"][3]["value"] = 1
    ok["values"][4]["shape"] = [1, 8]
    lifted = programs.batch_lift(ok, 3)
    assert lifted["values"][4]["shape"] == [3, 8]
    assert lifted["memoryPlan"]["pools"][2]["size"] == 3 * 8 * 4


def test_respatial_depthart_256():
    prog = load("depthart", "program-fp16.json")
    p = programs.respatial(prog, 256, 256)
    v = p["values"]
    assert v[p["inputIds"][0]]["shape"] == [1, 3, 256, 256]
    assert v[p["outputIds"][0]]["shape"] == [1, 1, 256, 256]
    sizes = [v[op["args"][1]]["items"] for op in p["chain"]
             if op["name"] == "aten.upsample_bilinear2d.vec" and v[op["args"][1]]["type"] == "list"]
    assert sizes == [[16, 16], [32, 32], [64, 64], [256, 256]]
    # every activation is 448/256 = 7/4 smaller on each side
    for a, b in zip(prog["values"], v):
        if a["type"] == "tensor" and a.get("weightsOffset") is None and len(a["shape"]) == 4:
            assert b["shape"][2] * 7 == a["shape"][2] * 4
    lifted = programs.batch_lift(p, 8)
    assert lifted["values"][lifted["outputIds"][0]]["shape"] == [8, 1, 256, 256]


def test_random_init_is_seeded_and_keeps_other_constants():
    prog, w = load("yolo26n", "program-fp16.json"), load("yolo26n", "weights-fp16.bin")
    a = programs.random_init(prog, w, seed=0)
    assert a == programs.random_init(prog, w, seed=0)
    assert a != programs.random_init(prog, w, seed=1)
    assert len(a) == len(w)
    v = prog["values"]
    for op in prog["chain"]:
        if op["name"] == "et_vk.prepack.default":
            c = v[op["args"][0]]
            o, n = c["weightsOffset"], c["weightsLength"]
            assert a[o:o + n] == w[o:o + n]
    conv = next(op for op in prog["chain"] if op["name"] == "aten.convolution.default")
    wt = v[conv["args"][1]]
    x = np.frombuffer(a[wt["weightsOffset"]:wt["weightsOffset"] + wt["weightsLength"]], np.float16)
    fan_in = int(np.prod(wt["shape"][1:]))
    assert abs(float(x.astype(np.float64).std()) - (2.0 / fan_in) ** 0.5) < 0.3 * (2.0 / fan_in) ** 0.5
