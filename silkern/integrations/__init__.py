"""Alias of :mod:`silkern_b200.integrations`."""
