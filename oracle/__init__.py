"""CPU oracle for the fused latent expert FFN.

TEST INFRASTRUCTURE ONLY.  Nothing in ``latent_b200`` imports this package;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and reference legs use it, and only as the checker / the timed CPU
restatement of the reference runtime.  The product path is the CUDA library
and fails loudly when that library is missing.

Parity pinning: every function in :mod:`oracle.latent_oracle` is checked
against golden vectors produced by the reference's own Python runtime
(``tests/golden/make_golden.py`` imports ``loader/latent_loader.py`` and
``loader/latent_runtime.py`` from the reference checkout and records inputs
and outputs as ``tests/golden/*.npz``).
"""

from .latent_oracle import *  # noqa: F401,F403
