"""Einshard notation front-end: data model, parser and axis families."""

from .spec import (
    Axes,
    Axis,
    AxisGroup,
    EllipsisAxis,
    GradAnnotation,
    InitSyncAnnotation,
    TensorAnnotation,
    TensorSpec,
)
from .parser import parse_sharding, sharding
from .families import cached_expand_axis_families, expand_axis_families, expand_family_mapping
