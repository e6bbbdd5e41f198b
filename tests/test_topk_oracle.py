"""CPU tests of the top-k oracle against torch.topk, the validator of the reference's tests
(roofline/workloads/hpcops_topk_cluster8.yaml: `reference: torch.topk on the CPU`)."""
import numpy as np


def test_oracle_matches_torch_topk(orc):
    import torch

    g = np.random.default_rng(1)
    cases = [g.standard_normal((4, 3000)).astype(np.float32),
             g.integers(0, 5, (3, 2000)).astype(np.float32),
             np.array([[np.inf, -np.inf, 0.0, -0.0, 1.0, np.nan, -1.0, np.nan]], np.float32)]
    for x in cases:
        for k in (1, 7, x.shape[1]):
            ref = torch.topk(torch.from_numpy(x), k, dim=1).values.numpy()
            got = orc.topk_values(x, k)
            assert np.array_equal(got, ref, equal_nan=True), (x.shape, k)
