"""Alias of :mod:`silkern_b200.kernels`."""

from silkern_b200.kernels import localize_hierarchical, localize_rowwise  # noqa: F401
