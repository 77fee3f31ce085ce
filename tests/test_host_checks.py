"""Host-side argument checks of the Python boundary (no GPU needed): the
kernels read caller buffers through raw pointers, so malformed masks and
output buffers must be refused before any launch."""
import pytest

torch = pytest.importorskip("torch")

from miniserve_b200.sampler import check_mask, check_out  # noqa: E402

CPU = torch.device("cpu")


def test_mask_must_be_cuda_32bit_words():
    for bad in (torch.zeros(2, 4, dtype=torch.uint8), torch.zeros(2, 4, dtype=torch.int64),
                torch.zeros(2, 4, dtype=torch.int32), [[0, 0]]):
        with pytest.raises(TypeError):
            check_mask(bad, 2, 100, CPU)


def test_out_buffers_checked():
    B = 3
    good = (torch.zeros(B, dtype=torch.int64), torch.zeros(B, dtype=torch.float32),
            torch.zeros(B, dtype=torch.int32))
    assert check_out(good, B, CPU) == good
    with pytest.raises(TypeError):
        check_out((good[0], torch.zeros(B, dtype=torch.float64), good[2]), B, CPU)
    with pytest.raises(TypeError):
        check_out((good[0].to(torch.int32), good[1], good[2]), B, CPU)
    with pytest.raises(ValueError):
        check_out((torch.zeros(B - 1, dtype=torch.int64), good[1], good[2]), B, CPU)
    with pytest.raises(ValueError):
        check_out((good[0], torch.zeros(2 * B, dtype=torch.float32)[::2], good[2]), B, CPU)
    with pytest.raises(TypeError):
        check_out(good[:2], B, CPU)
