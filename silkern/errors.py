"""Alias of :mod:`silkern_b200.errors`."""

from silkern_b200.errors import LocalizationError  # noqa: F401
