"""delrec (B200 edition): DelRec's delay-LIF layers and model zoo on hand-written sm_100a
CUDA kernels (libdelrec_b200.so).  Drop-in module API of the reference package
``delrec``: ``delrec.delay_layers``, ``delrec.networks``, ``delrec.utils``."""

__version__ = "1.0.0+b200"
