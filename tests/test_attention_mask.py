"""Host-side validation of the attention mask (no GPU): the decoder layer
honours a 2D left-padding key mask and refuses every other form."""
import pytest
import torch

from nki_moe_7013_b200.attention import left_padding


def test_no_mask_means_no_padding():
    assert left_padding(None, 2, 5, [0, 0]) is None


def test_left_padding_counts():
    m = torch.tensor([[1, 1, 1, 1], [0, 0, 1, 1], [0, 0, 0, 0]])
    assert left_padding(m, 3, 4, [0, 0, 0]) == [0, 2, 4]
    # a mask over cached + new tokens
    assert left_padding(torch.tensor([[0, 1, 1, 1, 1]]), 1, 2, [3]) == [1]


@pytest.mark.parametrize("mask", [
    torch.tensor([[1, 1, 0, 0]]),        # right padding
    torch.tensor([[1, 0, 1, 1]]),        # a hole
    torch.ones(1, 1, 4, 4),              # 4D mask
])
def test_other_masks_are_refused(mask):
    with pytest.raises(ValueError):
        left_padding(mask, 1, 4, [0])


def test_mask_must_cover_cache_and_new_tokens():
    with pytest.raises(ValueError):
        left_padding(torch.ones(1, 4), 1, 4, [2])
    with pytest.raises(ValueError):
        left_padding(torch.ones(2, 4), 1, 4, [0])
