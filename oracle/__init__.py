"""CPU oracle of the gated delta rule (test infrastructure; see oracle.py)."""
