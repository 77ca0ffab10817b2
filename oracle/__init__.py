"""CPU oracle (test infrastructure only); see oracle.py and forward_ref.cpp."""
