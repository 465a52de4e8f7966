"""pymolecular_b200 — B200-native EGNN layer (forward + backward over a dst-sorted CSR).

Drop-in for SatxaFortuny/PyMolecular ``models/EGNN/egnn_clean.py``:
``EGNN`` and ``E_GCL`` keep the reference constructor arguments, parameter
names and forward signatures; the math runs in hand-written sm_100a kernels
behind the C ABI of ``libegnn_b200.so`` (``include/egnn_b200.h``).
"""
from . import builders, losses
from .csr import CSR
from .egnn import E_GCL, EGNN, linear
from .losses import graph_sum_mse

__version__ = "0.1.0"
__all__ = ["CSR", "E_GCL", "EGNN", "builders", "graph_sum_mse", "linear", "losses"]
