"""Chains over more than 2^31 elements (64-bit element offsets in every
kernel that takes them): x[32768, 65540] fp32, 8.6 GB, through the C-ABI.

At this size the oracle's loops would take minutes, so the checks are the
size-independent properties of the ops: relu is bit-exact against
(0 < x) ? x : 0 evaluated element-wise on the device, and the full sum and
the column sums of relu(x) are within 1e-5 of fp64 sums of the kernel's own
stored values (relative to the sum of magnitudes). The data is generated on
the device (torch, plumbing only)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, COLS = 32768, 65540  # 2,147,614,720 elements > 2^31


@pytest.fixture(scope="module")
def big(ttc):
    import torch

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(29)
    x = torch.rand(ROWS, COLS, device="cuda", generator=g) * 2 - 1
    y = torch.empty_like(x)
    yield torch, x, y
    del x, y
    torch.cuda.empty_cache()


def test_relu_store_and_full_sum_past_2_to_31_elements(ttc, big):
    torch, x, y = big
    s = torch.empty(1, device="cuda")
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_RELU), ttc.instr(ttc.OP_STORE, idx=0)]
    d = ttc.chain_desc(ROWS, COLS, [ttc.in_view(x.data_ptr(), COLS)], [ttc.out_view(y.data_ptr(), COLS)], prog,
                       reduce=ttc.REDUCE_ALL, reduce_out=s.data_ptr())
    torch.cuda.synchronize()
    ttc.eltwise_chain(d)
    ttc.synchronize()
    want = torch.where(x > 0, x, torch.zeros((), device="cuda"))
    assert torch.equal(y.view(torch.int32), want.view(torch.int32))
    exact = float(y.double().sum())
    assert abs(float(s[0]) - exact) <= 1e-5 * exact
    # the last row, where 32-bit element offsets would have wrapped
    assert torch.equal(y[-1], want[-1])


def test_column_sums_past_2_to_31_elements(ttc, big):
    torch, x, y = big
    cs = torch.empty(COLS, device="cuda")
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_RELU)]
    d = ttc.chain_desc(ROWS, COLS, [ttc.in_view(x.data_ptr(), COLS)], [], prog, reduce=ttc.REDUCE_COLS,
                       reduce_out=cs.data_ptr())
    torch.cuda.synchronize()
    ttc.eltwise_chain(d)
    ttc.synchronize()
    r = torch.where(x > 0, x, torch.zeros((), device="cuda")).double()
    exact = r.sum(0)
    scale = r.abs().sum(0) + 1e-30
    err = ((cs.double() - exact).abs() / scale).max()
    assert float(err) <= 1e-5, float(err)
    assert np.isfinite(cs.cpu().numpy()).all()
