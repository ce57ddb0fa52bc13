"""CPU oracle for the depthwise path (test infrastructure only; see oracle.py)."""
