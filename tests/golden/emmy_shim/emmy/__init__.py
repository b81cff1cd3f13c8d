"""Test-only stand-in for the ``emmy`` package: just enough for the reference emitter to import."""
