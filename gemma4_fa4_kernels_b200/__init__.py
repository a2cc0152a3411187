"""B200-native (sm_100a) Gemma-4 attention backend.

Drop-in for the operator surface of the reference ``gemma4_fa4`` package:
the fixed-BSHD and packed-THD local-d256 / global-d512 adapters, the exact
mask builders and the Transformers backend registration.  Compute runs in
``libgemma4_b200.so`` (hand-written tcgen05/TMA kernels); there is no CPU or
library fallback.
"""

from .errors import GlobalBackwardBudgetExceeded, UnsupportedB200Path, UnsupportedH100Path

__all__ = ["GlobalBackwardBudgetExceeded", "UnsupportedB200Path", "UnsupportedH100Path"]
