"""Layer namespace with the reference's ``mamformer.layers`` names (re-exports ``models``)."""

from mamformer_b200.models import *  # noqa: F401,F403
from mamformer_b200.models import __all__  # noqa: F401
