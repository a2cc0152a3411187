"""Exception types of the operator surface.

They mirror the reference's fail-closed admission errors
(``src/gemma4_fa4/h100.py:37-42``): malformed inputs raise ``ValueError``;
inputs outside the supported contract raise ``UnsupportedB200Path``; a global
backward that the guarded HBM budget cannot admit raises
``GlobalBackwardBudgetExceeded`` before any launch.  ``UnsupportedH100Path``
is kept as an alias so callers written against the reference keep working.
"""


class UnsupportedB200Path(RuntimeError):
    """Raised when an input would leave the validated B200 contract."""


class GlobalBackwardBudgetExceeded(UnsupportedB200Path):
    """Raised before launch when guarded HBM cannot admit global backward."""


UnsupportedH100Path = UnsupportedB200Path
