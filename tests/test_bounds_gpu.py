"""Index checks of the gather / scatter kernels, with canary-padded buffers.

Every kernel that follows an index table (expert rows, slot positions, top-k ids) checks
each index against its range; a bad one records "index out of bounds" in the device error
word (``check_errors`` raises) and the access is skipped.  Each test hands a kernel one
index just past the end.  The operand and output tensors are views into larger buffers
whose extra rows hold a canary pattern: even an unchecked access would stay inside the
allocation, and the canary proves that no write went past the end.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

CANARY = -7.0


def _canaried(rows: int, cols: int, dev, pad: int = 4, dtype=torch.bfloat16):
    full = torch.full((rows + pad, cols), CANARY, dtype=dtype, device=dev)
    return full, full[:rows]


def _expect_bounds_error(dev):
    from saint_llm_b200.ops import gemm

    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="out of bounds"):
        gemm.check_errors(dev)
    gemm.check_errors(dev)  # cleared


def test_gather_rows_rejects_token_past_end(cuda):
    from saint_llm_b200.ops import backend, gemm

    T, D = 6, 256
    hfull, h = _canaried(T, D, cuda)
    h.copy_(torch.randn(T, D, device=cuda))
    row_token = torch.tensor([0, 5, -1, T, 2], dtype=torch.int32, device=cuda)  # T is one past the end
    out = torch.empty(5, D, dtype=torch.bfloat16, device=cuda)
    backend.ext().moe_gather(h, row_token, out, gemm.error_word(cuda))
    _expect_bounds_error(cuda)
    assert torch.equal(out[0], h[0]) and torch.equal(out[1], h[5]) and torch.equal(out[4], h[2])
    assert torch.count_nonzero(out[2]) == 0 and torch.count_nonzero(out[3]) == 0  # padding / rejected rows


def test_combine_and_backward_reject_position_past_end(cuda):
    from saint_llm_b200.ops import backend, gemm

    R, D, T, k = 8, 128, 3, 2
    y = torch.randn(R, D, device=cuda).to(torch.bfloat16)
    pos = torch.tensor([[0, 1], [2, R], [3, 4]], dtype=torch.int32, device=cuda)  # R is one past the end
    w = torch.rand(T, k, device=cuda)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=cuda)
    backend.ext().moe_combine(y, pos, w, out, gemm.error_word(cuda))
    _expect_bounds_error(cuda)
    want = torch.stack([w[0, 0] * y[0].float() + w[0, 1] * y[1].float(), w[1, 0] * y[2].float(),
                        w[2, 0] * y[3].float() + w[2, 1] * y[4].float()])
    torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-2)

    dout = torch.randn(T, D, device=cuda).to(torch.bfloat16)
    dyfull, dy = _canaried(R, D, cuda)
    dw = torch.full((T, k), 99.0, device=cuda)
    backend.ext().moe_combine_bwd(dout, y, pos, w, dy, dw, gemm.error_word(cuda))
    _expect_bounds_error(cuda)
    assert torch.all(dyfull[R:] == CANARY), "a write went past the end of dy"
    assert dw[1, 1].item() == 0.0
    torch.testing.assert_close(dw[0, 0], (dout[0].float() * y[0].float()).sum(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dy[2].float(), (w[1, 0] * dout[1].float()), rtol=2e-2, atol=2e-2)


def test_csa_select_mask_rejects_block_past_end(cuda):
    from saint_llm_b200.ops import backend, gemm

    n = 40
    top = torch.tensor([[[0, 39, -1, n]]], dtype=torch.int64, device=cuda)
    sel = torch.empty(1, 1, 2, dtype=torch.int32, device=cuda)
    backend.ext().csa_select_mask(top, n, sel, gemm.error_word(cuda))
    _expect_bounds_error(cuda)
    bits = sel.view(torch.int32).cpu().view(-1).tolist()
    assert bits[0] == 1 and (bits[1] & 0xFFFFFFFF) == (1 << 7), bits


def test_valid_indices_leave_error_word_clear(cuda):
    from saint_llm_b200.ops import backend, gemm

    T, D = 4, 128
    h = torch.randn(T, D, device=cuda).to(torch.bfloat16)
    row_token = torch.tensor([3, -1, 0], dtype=torch.int32, device=cuda)
    out = torch.empty(3, D, dtype=torch.bfloat16, device=cuda)
    backend.ext().moe_gather(h, row_token, out, gemm.error_word(cuda))
    torch.cuda.synchronize()
    gemm.check_errors(cuda)
    assert torch.equal(out[0], h[3]) and torch.equal(out[2], h[0])
