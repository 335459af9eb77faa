"""Training-metadata gradient targets (training.py) on CPU tensors: the
means2d leaf's per-view blocks, including views with no Gaussians."""

import torch

from dsl_splat_b200.training import ScreenGradientTarget


def _targets(views: int, n: int):
    leaf = torch.zeros(views, n, 2, requires_grad=True)
    fresh = {"count": views}
    return leaf, [ScreenGradientTarget(leaf, index=i, fresh=fresh) for i in range(views)]


def test_direct_buffers_are_the_views_blocks():
    leaf, targets = _targets(3, 4)
    blocks = [t.direct_buffer() for t in targets]
    for i, block in enumerate(blocks):
        block += i + 1  # what the render backward does in place
    assert torch.equal(leaf.grad[:, 0, 0], torch.tensor([1.0, 2.0, 3.0]))
    # a second backward through the same view adds instead of reusing the block
    assert targets[1].direct_buffer() is None
    targets[1].add(torch.ones(4, 2))
    assert torch.equal(leaf.grad[1], torch.full((4, 2), 3.0))


def test_views_without_gaussians():
    leaf, targets = _targets(2, 0)
    block = targets[0].direct_buffer()
    assert block is not None and block.shape == (0, 2)
    targets[1].add(torch.zeros(0, 2))
    assert leaf.grad.shape == (2, 0, 2)


def test_packed_rows_gather_the_visible_gaussians():
    # two views packed into one (5, 2) leaf: view 0 sees Gaussians 2 and 0,
    # view 1 sees Gaussians 1, 3 and 2 of a 4-Gaussian scene
    leaf = torch.zeros(5, 2, requires_grad=True)
    screen = torch.arange(8, dtype=torch.float32).view(4, 2)
    views = [(torch.tensor([2, 0]), 0, 2), (torch.tensor([1, 3, 2]), 2, 5)]
    for ids, begin, end in views:
        target = ScreenGradientTarget(leaf, gaussian_ids=ids, begin=begin, end=end)
        assert target.direct_buffer() is None
        target.add(screen)
        target.add(screen)
    expected = 2 * torch.cat([screen[ids] for ids, _, _ in views])
    assert torch.equal(leaf.grad, expected)
