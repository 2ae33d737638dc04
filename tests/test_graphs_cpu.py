"""Row-bucket selection of the per-bucket CUDA graphs (no GPU): the reference's
decode and prefill buckets (crates/glm-cli/src/profile.rs:10-11)."""
import pytest

from glmaxx_b200.graphs import DECODE_ROWS, PREFILL_ROWS, bucket_for


def test_reference_buckets():
    assert DECODE_ROWS == (1, 2, 4, 8, 16, 32, 64, 128)
    assert PREFILL_ROWS == (256, 512, 1024, 2048, 3072)


@pytest.mark.parametrize("rows,bucket", [(1, 1), (3, 4), (64, 64), (65, 128), (128, 128),
                                         (129, 256), (300, 512), (2049, 3072), (3072, 3072)])
def test_bucket_for(rows, bucket):
    assert bucket_for(rows) == bucket


def test_bucket_limits():
    with pytest.raises(ValueError):
        bucket_for(0)
    with pytest.raises(ValueError):
        bucket_for(3073)
    assert bucket_for(5, (8, 2)) == 8
