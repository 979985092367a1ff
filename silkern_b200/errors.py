"""The one exception type every public entry point raises."""

from __future__ import annotations


class LocalizationError(ValueError):
    """An invalid localization configuration, geometry or buffer binding.

    Entry points fail closed: they raise this before anything is launched
    instead of falling back to another code path (silkern/errors.py:6-11 in
    the reference defines the same convention).
    """
