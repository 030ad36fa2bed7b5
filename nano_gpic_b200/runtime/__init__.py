"""Execution helpers around the model: CUDA-graph replay of launch-bound forwards (graphs.py)."""
