"""Argument checks of the Python mirror that need no GPU: buffers must be
device memory of the right element type, or raw device pointers."""
import pytest
import torch

from ark_b200.optimizer import _ptr


def test_raw_pointers_and_none_pass_through():
    assert _ptr(None, "f16") is None
    assert _ptr(0x7F0000001000, "f32") == 0x7F0000001000


def test_host_tensors_and_other_objects_are_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        _ptr(torch.zeros(8, dtype=torch.float16), "f16")
    with pytest.raises(TypeError):
        _ptr([0.0] * 8, "f32")
