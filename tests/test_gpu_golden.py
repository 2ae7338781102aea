"""The kernel (through the C ABI) against the reference's golden fixtures."""
import numpy as np
import pytest
import torch

from tests import golden_cases
from tests.helpers import LSE_RTOL, O_ATOL, run_capi

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_cases.case_names())
@pytest.mark.parametrize("out_f32", [False, True])
def test_kernel_matches_reference_fixture(name, out_f32):
    c = golden_cases.load(name)
    o, lse = run_capi(c["q"], c["k"], c["v"], torch.from_numpy(c["sel"]), l_prime=c["LP"], BQ=c["BQ"],
                      out_f32=out_f32)
    torch.cuda.synchronize()
    o = o.float().cpu().numpy().astype(np.float64)
    got = golden_cases.rows_of(o, c["rows"])
    assert np.abs(got - c["o_rows"]).max() <= O_ATOL
    # every element through the full-tensor checksums (bf16 output rounding bounds their drift)
    cs = golden_cases.checksums(o)
    scale = np.abs(c["checksums"]) + o.size ** 0.5
    assert (np.abs(cs - c["checksums"]) <= 2e-3 * scale).all(), (cs, c["checksums"])
    l = lse.cpu().numpy().astype(np.float64)
    fin = np.isfinite(c["lse"])
    assert (np.isneginf(l) == ~fin).all()
    assert (np.abs(l[fin] - c["lse"][fin]) / np.maximum(np.abs(c["lse"][fin]), 1.0)).max() <= LSE_RTOL
