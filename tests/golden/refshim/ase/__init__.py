"""Minimal stand-in of the ASE modules the reference imports at module level
(test infrastructure only; the fixture generator never calls the ASE
calculator or neighbour-list machinery, it calls the reference's step
functions directly with a neighbour list built by the test oracle)."""
