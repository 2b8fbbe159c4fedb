"""torch.ops.aegis.matmul without a GPU: the op is registered, its fake
implementation gives the output shape and dtype under meta tensors and
rejects mismatched shapes, and operand layouts are read from strides."""
import pytest
import torch

import aegis_capi as ac
import aegis_torch


def test_registered_and_fake_shapes():
    a = torch.empty(64, 48, dtype=torch.bfloat16, device="meta")
    b = torch.empty(48, 80, dtype=torch.bfloat16, device="meta")
    c = torch.ops.aegis.matmul(a, b)
    assert c.shape == (64, 80) and c.dtype == torch.bfloat16 and c.device.type == "meta"
    with pytest.raises(Exception):
        torch.ops.aegis.matmul(a, torch.empty(47, 80, dtype=torch.bfloat16, device="meta"))


def test_operand_layouts_from_strides():
    t = torch.empty(6, 10, dtype=torch.float16)
    assert aegis_torch._operand(t)[1:] == (ac.ROW_MAJOR, 10)
    assert aegis_torch._operand(t.t())[1:] == (ac.COL_MAJOR, 10)  # a 10 x 6 column-major view
    sub = t[:, :8]                                                # padded rows: ld 10
    assert aegis_torch._operand(sub)[1:] == (ac.ROW_MAJOR, 10)
    odd = t[::2, ::2]                                             # neither: copied
    got, lay, ld = aegis_torch._operand(odd)
    assert got.is_contiguous() and (lay, ld) == (ac.ROW_MAJOR, 5)
