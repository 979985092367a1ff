"""Alias of :mod:`silkern_b200.verify`."""

from silkern_b200.verify import (  # noqa: F401
    CHECKS,
    DEFAULT_MATRIX,
    DETERMINISM_REPEATS,
    GUARD_ELEMENTS,
    REPLAY_COUNT,
    CellReport,
    ConformanceReport,
    _expected_order,
    _random_case,
    conformance,
    main,
    replay_gate,
)
