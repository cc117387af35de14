"""Device-side data generation: the quantizers match the oracle bit for bit (Q4_K is the
reference quantizer, q4k.rs:85-160), and the device normal generator follows the oracle's
seeded stream."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t", [oracle.Q4_K, oracle.Q6_K, oracle.Q8_0])
def test_device_quantizer_bit_exact(engine, t):
    n = 256 * 4096
    x = oracle.normal(42 + t, n, 0.0, 0.02)
    x[:256] = 0.0  # an all-zero block
    x[256:512] = np.linspace(-3, 3, 256, dtype=np.float32)
    ref = oracle.quantize(t, x)
    xd = torch.from_numpy(x).cuda()
    q = torch.empty(ref.size, dtype=torch.uint8, device="cuda")
    engine.set_stream(torch.cuda.current_stream())
    try:
        engine.quantize_dev(t, xd, q)
        torch.cuda.synchronize()
    finally:
        engine.set_stream(None)
    assert np.array_equal(ref, q.cpu().numpy())


def test_device_normal_follows_oracle_stream(engine):
    n = 1 << 20
    ref = oracle.normal(7, n, 0.0, 0.02)
    out = torch.empty(n, device="cuda")
    engine.set_stream(torch.cuda.current_stream())
    try:
        engine.synth_normal_dev(7, out, 0.0, 0.02)
        torch.cuda.synchronize()
    finally:
        engine.set_stream(None)
    got = out.cpu().numpy()
    # identical up to last-bit differences of double log/sin/cos
    assert np.abs(got - ref).max() <= 1e-7
    assert np.mean(got == ref) > 0.99
