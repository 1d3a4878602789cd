"""GPU parity: HACCmk's short-range force step (a3b_haccmk_step10) against the oracle, which equals the benchmark's own
CPU gold bit for bit (tests/test_oracle.py). The kernel sums each target's pairs in another order than the gold's
sequential loop and uses the MUFU reciprocal square root, so the check is normwise: max |error| / max |value| per
component <= 1e-5."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n2,n1", [(15000, 784), (1000, 1000), (4096, 100), (15001 + 3, 5), (64, 1)])
def test_haccmk_step10_vs_oracle(cuda, port, n2, n1):
    from alpaka3_b200 import algo
    xx, yy, zz, m = port.haccmk_init(n2)
    want = port.haccmk_step10(n1, xx, yy, zz, m)
    T = [torch.from_numpy(a).to(cuda) for a in (xx, yy, zz, m)]
    V = [torch.full((n1,), 7.0, dtype=torch.float32, device=cuda) for _ in range(3)]
    algo.haccmk_step10(*T, *V, n1, 0.5, 0.03, 0.23)
    torch.cuda.synchronize()
    for v, w in zip(V, want):
        got = v.cpu().numpy()
        rel = float(np.max(np.abs(got - w)) / np.max(np.abs(w)))
        assert rel <= 1e-5, rel


def test_haccmk_deterministic(cuda, port):
    from alpaka3_b200 import algo
    xx, yy, zz, m = port.haccmk_init(15000)
    T = [torch.from_numpy(a).to(cuda) for a in (xx, yy, zz, m)]
    runs = []
    for _ in range(3):
        V = [torch.zeros(784, dtype=torch.float32, device=cuda) for _ in range(3)]
        algo.haccmk_step10(*T, *V, 784, 0.5, 0.03, 0.23)
        runs.append(torch.cat(V).cpu())
    assert all(torch.equal(runs[0], r) for r in runs[1:])
