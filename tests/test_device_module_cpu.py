"""The torch.mcpu module's seeding on the host: mcpu tensors are drawn by the
host generator, so torch.manual_seed (which also calls the registered device
module's manual_seed_all) and torch.mcpu.manual_seed must seed it, once, with
no recursion between the two."""

import torch


def test_manual_seed_does_not_recurse_and_seeds_the_host_generator():
    import torch_mcpu_b200.device  # noqa: F401  registers torch.mcpu

    torch.manual_seed(123)
    a = torch.randn(5)
    torch.mcpu.manual_seed(123)
    b = torch.randn(5)
    torch.mcpu.manual_seed_all(123)
    c = torch.randn(5)
    assert torch.equal(a, b) and torch.equal(a, c)
