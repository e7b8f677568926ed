"""Output-shape helpers shared by the tests (no oracle or engine code)."""


def _hw(v):
    v = list(v) if isinstance(v, (list, tuple)) else [v]
    return (v[0], v[0]) if len(v) == 1 else (v[0], v[1])


def conv_out_shape(xshape, wshape, p):
    B, IC, IH, IW = xshape
    OC, _, KH, KW = wshape
    s, pd, d = _hw(p["stride"]), _hw(p["padding"]), _hw(p["dilation"])
    OH = (IH + 2 * pd[0] - d[0] * (KH - 1) - 1) // s[0] + 1
    OW = (IW + 2 * pd[1] - d[1] * (KW - 1) - 1) // s[1] + 1
    return [B, OC, OH, OW]


def convT_out_shape(xshape, wshape, p):
    B, IC, IH, IW = xshape
    _, ocpg, KH, KW = wshape
    s, pd, d, op = (_hw(p["stride"]), _hw(p["padding"]), _hw(p["dilation"]),
                    _hw(p["output_padding"]))
    OH = (IH - 1) * s[0] - 2 * pd[0] + d[0] * (KH - 1) + op[0] + 1
    OW = (IW - 1) * s[1] - 2 * pd[1] + d[1] * (KW - 1) + op[1] + 1
    return [B, ocpg * p["groups"], OH, OW]
