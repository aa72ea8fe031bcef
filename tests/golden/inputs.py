"""Seeded synthetic inputs shared by the golden generator, tests and bench.

CPU ``torch.Generator`` streams are deterministic across machines, so the
fixtures store only reference outputs and these functions rebuild inputs.
"""
import torch


def qk_inputs(seed, shape, dtype, k_offset_std=0.0, outliers=0.0):
    """Q,K,V ~ N(0,1); K plus a per-(b,h,channel) offset ~ N(0, k_offset_std^2);
    optionally a Bernoulli(outliers) mask of Q/K entries scaled x20."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(*shape, generator=g)
    k = torch.randn(*shape, generator=g)
    if k_offset_std:
        k = k + torch.randn(shape[0], shape[1], 1, shape[3], generator=g) * k_offset_std
    if outliers:
        for t in (q, k):
            m = torch.rand(*shape, generator=g) < outliers
            t[m] *= 20
    v = torch.randn(*shape, generator=g)
    return q.to(dtype), k.to(dtype), v.to(dtype)


def mixture_values(seed, shape, dtype, centroids=16, centroid_std=2 ** 0.5, within_std=0.3):
    """V from a Gaussian mixture: centroids ~ N(0, centroid_std^2) per channel,
    within-cluster std ``within_std``, labels uniform (tokens randomly ordered)."""
    g = torch.Generator().manual_seed(seed + 100)
    cent = torch.randn(shape[0], shape[1], centroids, shape[3], generator=g) * centroid_std
    lab = torch.randint(0, centroids, tuple(shape[:3]), generator=g)
    v = cent.gather(2, lab.unsqueeze(-1).expand(*shape)) + within_std * torch.randn(*shape, generator=g)
    return v.to(dtype)
