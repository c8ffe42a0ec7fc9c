"""The SHA-256 leaf kernel against hashlib on the host: every leaf digest of
buffers of several sizes (whole leaves, a short last leaf, a tail that is not
a multiple of 64 bytes, a buffer that does not start on 16 bytes) is the
SHA-256 of the same bytes, so the GPU tree digest equals the host one."""
import pytest
import torch

from shift_b200.utils.digest import LEAF, leaf_digests, sha256tree

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes", [64, 100, LEAF, 3 * LEAF + 55, 5 * LEAF + 56, 7 * LEAF + 119])
def test_leaves_match_hashlib(nbytes):
    g = torch.Generator().manual_seed(nbytes)
    host = torch.randint(0, 256, (nbytes,), generator=g, dtype=torch.uint8)
    dev = host.cuda()
    assert leaf_digests(dev) == leaf_digests(host)
    assert sha256tree(dev) == sha256tree(host)


def test_unaligned_start_and_fp32_state():
    host = torch.randint(0, 256, (2 * LEAF + 77,), dtype=torch.uint8)
    dev = host.cuda()
    assert leaf_digests(dev[3:]) == leaf_digests(host[3:])           # byte-loaded path
    x = torch.randn(1 << 20, device="cuda")
    assert sha256tree(x) == sha256tree(x.cpu())
    y = x.clone()
    y[12345] = torch.nextafter(y[12345], torch.tensor(float("inf"), device="cuda"))
    assert sha256tree(y) != sha256tree(x)
