"""Stand-in ``emmy`` package for running the reference compiler (test infrastructure)."""
