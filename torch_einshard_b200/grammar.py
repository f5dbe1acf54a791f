"""Parser entry points (module path kept for users of ``es.grammar``).

Reference counterpart: ``src/torch_einshard/grammar.py`` (a parsley grammar
there; a hand-written parser here).
"""

from .notation.parser import parse_sharding, sharding  # noqa: F401
from .notation.spec import Axes, Axis, AxisGroup, EllipsisAxis, TensorAnnotation, TensorSpec  # noqa: F401
