"""Axis-family expansion (module path kept for users of ``es.families``)."""

from .notation.families import cached_expand_axis_families, expand_axis_families, expand_family_mapping  # noqa: F401
