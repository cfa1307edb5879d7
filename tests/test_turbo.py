"""TurboQuant host logic on CPU: matrices drawn as the reference draws them,
the reference's orthogonality tolerance, and the empty-cache contract
(kandiga tests/test_kv_compress.py: test_rotation_matrix_orthogonal,
test_empty_cache)."""
import numpy as np

from kandiga_b200.kv_compress import TurboQuantCache, turboquant_matrices
from oracle import oracle as O


def test_matrices_match_oracle_draw():
    for d, seed in ((128, 42), (64, 123)):
        r, p = turboquant_matrices(d, seed)
        ref = O.TurboQuantRef(d, 8, seed)
        assert np.array_equal(r, ref.rotation)
        assert np.array_equal(p, ref.qjl_proj)
        assert set(np.unique(np.abs(p) * np.sqrt(d)).round(6)) == {1.0}


def test_rotation_matrix_orthogonal():
    cache = TurboQuantCache(head_dim=128, num_heads=8)
    r = cache.rotation.numpy()
    np.testing.assert_allclose(r @ r.T, np.eye(128), atol=1e-5)
    assert np.array_equal(cache.rotation_t.numpy(), r.T)


def test_empty_cache():
    cache = TurboQuantCache(head_dim=128, num_heads=8)
    assert cache.keys is None
    assert cache.values is None
    assert cache.seq_len == 0
    assert cache.memory_bytes == 0
    assert cache.compression_ratio == 1.0
