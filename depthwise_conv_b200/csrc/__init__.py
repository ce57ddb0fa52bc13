"""CUDA sources of the engine and their build script (build.py)."""
