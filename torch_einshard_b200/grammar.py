"""Parser entry points (module path kept for users of ``es.grammar``)."""

from .notation.parser import parse_sharding, sharding  # noqa: F401
from .notation.spec import Axes, Axis, AxisGroup, EllipsisAxis, TensorAnnotation, TensorSpec  # noqa: F401
