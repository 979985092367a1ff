"""Alias of :mod:`silkern_b200.workspace`."""

from silkern_b200.workspace import workspace_shapes  # noqa: F401
