"""Axis-family expansion: a text rewrite applied before parsing.

``*spatial`` expands to the family's axes (``h w``); a bracketed zip
``[*spatial *window]`` expands to factored groups ``(h wh) (w ww)``.  Brackets
that hold parameter annotations (``[param, grad=...]``) are left untouched.
Mappings keyed by a family name (``sizes``, ``shifts``, ``halos``,
``windows``, ``padding``, FFT ``axes``) are expanded to one entry per axis.

Behaviour follows ``src/torch_einshard/families.py:44-136`` of the reference
(same error texts, same caching contract: cached results are copied before
being returned so callers may mutate them).
"""

import re
from functools import lru_cache

__all__ = [
    "expand_family_mapping",
    "expand_axis_families",
    "cached_expand_axis_families",
]

_FAMILY_REF = re.compile(r"\*([A-Za-z0-9]+)")
_BRACKETS = re.compile(r"\[([^\]]+)\]")
_ANNOTATION_PREFIXES = ("param", "grad=", "init_sync=")


def _families(families) -> dict:
    return {} if families is None else {name: tuple(axes) for name, axes in families.items()}


def _bare_axis_name(text: str) -> str:
    return text.split("/", 1)[0].strip()


def expand_family_mapping(mapping, families, *, label):
    """Expand family-name keys of ``mapping`` into per-axis keys.

    A scalar (or string) value is broadcast to every axis of the family; an
    iterable value must have one entry per axis.  Conflicting values for the
    same expanded axis are rejected.
    """
    families = _families(families)
    if not isinstance(mapping, dict) or not families:
        return mapping
    expanded = {}
    for key, value in mapping.items():
        if key not in families:
            expanded[key] = value
            continue
        members = families[key]
        if isinstance(value, (str, bytes)):
            values = (value,) * len(members)
        else:
            try:
                values = tuple(value)
            except TypeError:
                values = (value,) * len(members)
        if len(values) != len(members):
            raise ValueError(f"{label} family {key!r} has {len(values)} values for {len(members)} axes")
        for member, member_value in zip(members, values):
            axis = _bare_axis_name(member)
            if axis in expanded and expanded[axis] != member_value:
                raise ValueError(f"Conflicting {label.lower()} for expanded axis {axis!r}")
            expanded[axis] = member_value
    return expanded


def _holds_annotation(content: str) -> bool:
    entries = [re.sub(r"\s+", "", item) for item in content.split(",")]
    return bool(entries) and all(entry.startswith(_ANNOTATION_PREFIXES) for entry in entries)


def _zip_brackets(match, families) -> str:
    content = match.group(1)
    if _holds_annotation(content):
        return match.group(0)
    refs = content.split()
    if not refs or not all(ref.startswith("*") for ref in refs):
        raise ValueError("Zipped axis-family groups must contain only family references")
    names = [ref[1:] for ref in refs]
    for name in names:
        if name not in families:
            raise ValueError(f"Unknown axis family {name!r}")
    if len({len(families[name]) for name in names}) != 1:
        raise ValueError("Zipped axis families must have matching lengths")
    columns = zip(*(families[name] for name in names))
    return " ".join("(" + " ".join(column) + ")" for column in columns)


def expand_axis_families(expression, sizes=None, families=None):
    """Return ``(expanded_expression, expanded_sizes)``."""
    families = _families(families)
    if not families:
        return expression, sizes

    def single(match):
        name = match.group(1)
        if name not in families:
            raise ValueError(f"Unknown axis family {name!r}")
        return " ".join(families[name])

    expression = _BRACKETS.sub(lambda m: _zip_brackets(m, families), expression)
    expression = _FAMILY_REF.sub(single, expression)
    return expression, expand_family_mapping(sizes, families, label="Size")


def _freeze(mapping):
    if mapping is None or not isinstance(mapping, dict):
        return mapping
    return tuple(sorted(
        (key, tuple(value) if isinstance(value, (list, tuple)) else value)
        for key, value in mapping.items()
    ))


def _thaw(key):
    if isinstance(key, tuple):
        return dict(key)
    return key


@lru_cache(maxsize=1024)
def _expand_cached(expression, frozen_sizes, frozen_families):
    return expand_axis_families(expression, _thaw(frozen_sizes), dict(frozen_families))


def cached_expand_axis_families(expression, sizes=None, families=None):
    frozen_families = tuple(sorted(_families(families).items()))
    expanded, expanded_sizes = _expand_cached(expression, _freeze(sizes), frozen_families)
    if isinstance(expanded_sizes, dict):
        expanded_sizes = dict(expanded_sizes)
    elif isinstance(expanded_sizes, list):
        expanded_sizes = list(expanded_sizes)
    return expanded, expanded_sizes
