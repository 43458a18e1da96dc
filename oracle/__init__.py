"""CPU oracle (test infrastructure only); see dit_ref.py."""
