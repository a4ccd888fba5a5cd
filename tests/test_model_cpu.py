"""Host-side helpers of the model that need no GPU."""

import torch


def test_prefix_lengths_of_host_masks():
    from techjam_b200.model import prefix_lengths
    m = torch.zeros(3, 8, dtype=torch.bool)
    m[0, :5] = True
    m[1, :] = True
    assert prefix_lengths(m, 3, 8) == [5, 8, 0]
    assert prefix_lengths(m.to(torch.uint8), 3, 8) == [5, 8, 0]
    assert prefix_lengths(None, 2, 4) == [4, 4]
    m[2, 3] = True  # a hole: not a prefix, so forward_host uploads every row
    assert prefix_lengths(m, 3, 8) is None
