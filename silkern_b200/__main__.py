"""``python -m silkern_b200`` runs the conformance matrix on the local device."""

from silkern_b200.verify import main

raise SystemExit(main())
