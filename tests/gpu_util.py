"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch


def random_graph(n: int, e: int, seed: int, heavy: tuple[tuple[int, int], ...] = (),
                 dup_frac: float = 0.1, loops: int = 3) -> torch.Tensor:
    """edge_index [2,E] with duplicates, a few self-loops and optional heavy destinations."""
    g = torch.Generator().manual_seed(seed)
    ei = torch.randint(0, n, (2, e), generator=g)
    parts = [ei, ei[:, : int(e * dup_frac)]]
    for node, deg in heavy:
        src = torch.randint(0, n, (deg,), generator=g)
        parts.append(torch.stack([src, torch.full((deg,), node)]))
    if loops:
        v = torch.randint(0, n, (loops,), generator=g)
        parts.append(torch.stack([v, v]))
    return torch.cat(parts, dim=1)


def device_csr(ei: torch.Tensor, n: int, device, *, self_loops=True, dedupe=False):
    from gnnc.b200 import runtime as rt

    return rt.csr_from_coo(ei.to(device), n, self_loops=self_loops, dedupe=dedupe)


def assert_close(got: torch.Tensor, ref: torch.Tensor, rtol=1e-4, atol=1e-4):
    got = got.detach().double().cpu().numpy()
    ref = ref.detach().double().cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol)
