"""Drop-in import path of the reference package (``hopper_gmm_forward``).

Code written against the reference -- ``from hopper_gmm_forward import
hopper_gmm_fwd`` -- runs unchanged on the B200 implementation in
:mod:`gmm_b200`.
"""

from gmm_b200 import hopper_gmm_fwd  # noqa: F401

__all__ = ["hopper_gmm_fwd"]
