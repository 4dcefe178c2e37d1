"""Reference-compatible module API of the rotor-scan path.

Same import paths, names, signatures and state_dict keys as the reference's
``python`` package (python/clifford_scan.py, clifford_cl6.py, clifford_cl8.py,
clifford_layer.py, clifford_model.py).  The scan, Cayley rotor and cell run on the
CUDA library (csn_b200); everything else (projections, norms, heads) is PyTorch.
"""
