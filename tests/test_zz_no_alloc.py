"""nq_quantize_cols_noalloc: the per-column quantize for callers that cannot
allocate device memory during the call -- an engine whose allocator already
owns all of HBM, a plugin host that only passes input and output buffers, or
a loop that must not take cudaMalloc's implicit synchronisation.  Its scratch
is a fixed device array inside the library instead of pool memory.

Checked through the C ABI against nq_quantize_cols (bit-identical codes and
scales, the same bar as every quantize test here) on two calls in a row: the
second call uses smaller values, so scratch left over from the first call
would show up as wrong scales.  This file is collected last on purpose."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    return capi


def run(nq, fn, x, fmt, offset=0):
    from gpu_util import dev, empty, host, ptr, stream
    rows, cols = x.shape
    d_x, d_q, d_s = dev(x, offset), empty(rows * cols), empty(4 * cols)
    fn(ptr(d_x), ptr(d_q), ptr(d_s), rows, cols, fmt, stream())
    return host(d_q, np.uint8, (rows, cols)), host(d_s, np.float32)


@pytest.mark.parametrize("fmt", [0, 2])
def test_noalloc_matches_pooled_entry_point_twice(nq, fmt):
    rng = np.random.default_rng(42 + fmt)
    first = (rng.standard_normal((1024, 3000)) * 0.5).astype(np.float32)
    second = (rng.standard_normal((4096, 2500)) * 0.02).astype(np.float32)  # smaller amax everywhere
    for x in (first, second):
        q_new, s_new = run(nq, nq.quantize_cols_noalloc, x, fmt)
        q_ref, s_ref = run(nq, nq.quantize_cols, x, fmt)
        np.testing.assert_array_equal(s_new, s_ref)
        np.testing.assert_array_equal(q_new, q_ref)


@pytest.mark.parametrize("rows,cols,offset", [(37, 1027, 0), (19, 1027, 4), (3, 65536, 0)])
def test_noalloc_ragged_widths_and_the_limit(nq, rows, cols, offset):
    """Widths that are not a multiple of 4 (the kernels' scalar column tail),
    an unaligned source, and the largest width the fixed scratch holds."""
    rng = np.random.default_rng(rows * cols)
    for scale in (1.0, 0.01):   # two calls in a row, the second with smaller maxima
        x = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
        for fmt in (0, 2):
            q_new, s_new = run(nq, nq.quantize_cols_noalloc, x, fmt, offset)
            q_ref, s_ref = run(nq, nq.quantize_cols, x, fmt, offset)
            np.testing.assert_array_equal(s_new, s_ref)
            np.testing.assert_array_equal(q_new, q_ref)


def test_noalloc_rejects_widths_beyond_its_scratch(nq):
    from nova_b200.capi import NqError
    with pytest.raises(NqError, match="exceeds the fixed scratch of 65536"):
        nq.quantize_cols_noalloc(16, 16, 16, 2, 65537, 0, 0)
