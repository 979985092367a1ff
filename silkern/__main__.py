"""``python -m silkern`` runs the conformance matrix on the local device."""

from silkern_b200.verify import main

raise SystemExit(main())
