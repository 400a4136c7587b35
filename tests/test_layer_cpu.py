"""Host-side contract of the layers that needs no GPU: output shape and dtype
follow the reference's forward (moe_layer.py:519, ep.py:150)."""

import pytest
import torch

from reframework_b200.moe.moe_layer import reference_output


def test_output_shape_follows_the_reference():
    H = 8
    out = torch.randn(6, H, dtype=torch.bfloat16)
    assert reference_output(out, torch.empty(6, H), H).shape == (6, H)
    assert reference_output(out[:1], torch.empty(H), H).shape == (1, H)  # one [H] token -> [1, H]
    assert reference_output(out, torch.empty(6, 1, H), H).shape == (6, H)  # [B, 1, H] -> [B, H]
    assert reference_output(out[:0], torch.empty(0, H), H).shape == (0, H)
    with pytest.raises(RuntimeError):
        reference_output(out, torch.empty(3, 2, H), H)  # the reference's reshape rejects [B, S > 1, H]


def test_output_dtype_is_the_input_dtype():
    out = torch.randn(4, 8, dtype=torch.bfloat16)
    assert reference_output(out, torch.empty(4, 8, dtype=torch.float32), 8).dtype == torch.float32
    assert reference_output(out, torch.empty(4, 8, dtype=torch.bfloat16), 8).data_ptr() == out.data_ptr()  # no copy
