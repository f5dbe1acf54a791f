"""Axis-family expansion (module path kept for users of ``es.families``).

Reference counterpart: ``src/torch_einshard/families.py``.
"""

from .notation.families import cached_expand_axis_families, expand_axis_families, expand_family_mapping  # noqa: F401
