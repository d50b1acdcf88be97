"""invision_b200 -- B200 (sm_100a) dense-linear engine for Envision (hshatti/Invision).

The product is ``lib/libenvgemm.so`` (C ABI in ``include/envgemm.h``); ``envg`` is its Python
binding and a mirror of the reference's QNN operator names for this path.
"""
from . import envg  # noqa: F401
