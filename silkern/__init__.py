"""Drop-in name for :mod:`silkern_b200`.

Code written against the reference ``silkern`` package imports this one
unchanged: every public name (and the private helpers the reference's tests
use) resolves to the B200 implementation.
"""

from silkern_b200 import *  # noqa: F401,F403
from silkern_b200 import __all__, __version__, exact_stable_compact_reference  # noqa: F401
