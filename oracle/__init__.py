"""CPU oracle of the fused operators (test infrastructure, never a product path).

See gko_oracle.py for the reference formulas each function restates.
"""

from .gko_oracle import *  # noqa: F401,F403
from .gko_oracle import rel_err  # noqa: F401
