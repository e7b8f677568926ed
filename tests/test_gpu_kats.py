"""The reference's hot-path known-answer tests, run on the B200 engine
through the wgx API exactly as the reference drives WebGPU."""
import pytest

from kat_cases import cases, run_engine

CASES = cases()


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_reference_kat_on_engine(ctx, case):
    case.check(run_engine(ctx, case))
