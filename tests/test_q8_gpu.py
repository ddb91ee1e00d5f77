"""Q8_0 quantise/dequantise kernels against gguf-py's bytes (bit-exact)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_q8_0_quantize_many_ties(cuda):
    """4M weight-like values (the seeded N(0, 0.02) stream): products x * (1/d)
    that round to an exact .5 must round away from zero, as the reference does."""
    import torch
    from oracle import oracle as O
    from toy_b200._lib import lib
    x, _ = O.gaussian_fill(O.lcg_seed_state(11), 1 << 22, 0.02)
    rows, K = (1 << 22) // 512, 512
    want = O.q8_0_quantize(x.reshape(rows, K)).reshape(-1)
    xd = torch.from_numpy(x).to(cuda)
    q = torch.zeros(want.size, dtype=torch.uint8, device=cuda)
    assert lib().tb2_q8_0_quantize(xd.data_ptr(), q.data_ptr(), rows, K, None) == 0
    got = q.cpu().numpy()
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, (bad[:8], got[bad[:8]], want[bad[:8]])


@pytest.mark.parametrize("name", list("abcde"))
def test_q8_0_quantize_dequantize_bit_exact(cuda, name):
    import torch
    from toy_b200._lib import lib
    z = np.load(os.path.join(GOLD, "q8_0.npz"))
    x = z[name + "_x"]
    rows, K = x.shape
    xd = torch.from_numpy(x).to(cuda)
    q = torch.zeros(rows * K // 32 * 34, dtype=torch.uint8, device=cuda)
    assert lib().tb2_q8_0_quantize(xd.data_ptr(), q.data_ptr(), rows, K, None) == 0
    hi = torch.empty(rows * K, dtype=torch.bfloat16, device=cuda)
    lo = torch.empty_like(hi)
    f = torch.empty(rows * K, dtype=torch.float32, device=cuda)
    assert lib().tb2_q8_0_dequantize(q.data_ptr(), hi.data_ptr(), lo.data_ptr(), f.data_ptr(), rows, K, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), z[name + "_q"].reshape(-1))
    assert np.array_equal(f.cpu().numpy().view(np.uint32), z[name + "_dq"].reshape(-1).view(np.uint32))
