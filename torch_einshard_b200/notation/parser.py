"""Hand-written parser for einshard expressions.

Accepted language (the same one the reference accepts with its parsley PEG
grammar, ``src/torch_einshard/grammar.py:9-31``)::

    expr      := input [',' input] '->' output           (whole string, no trailing text)
    input     := axes [partial] [annotation]
    output    := axes [partial]
    axes      := (ws (group | '...' | axis))+
    axis      := ident [ws '/' ws mesh]
    group     := '(' (ws axis)+ ws ')'
    partial   := ws '//' ws (mesh | '(' ws mesh (ws ',' ws mesh)* ws ')')
    annotation:= ws '[' ws item (ws ',' ws item)* ws ']'
    item      := 'param' | 'grad' ws '=' ws value | 'init_sync' ws '=' ws value
    ident     := [A-Za-z0-9_]+          mesh := ident ('-' ident)*
    value     := ident ('-' ident)* [':' ident]

Whitespace is allowed before every axis, around ``/``, ``//``, ``,`` and ``->``,
but the expression must end right after the output spec.  The parser is a
single left-to-right scan with ordered-choice backtracking on a cursor; results
are LRU-cached by expression text and a fresh copy is handed out per call so
that callers may mutate the returned specs.
"""

from functools import lru_cache

from .spec import Axes, Axis, AxisGroup, EllipsisAxis, TensorAnnotation, TensorSpec

__all__ = ["parse_sharding", "sharding", "EinshardSyntaxError"]


class EinshardSyntaxError(Exception):
    """Raised by the scanner; :func:`parse_sharding` rewraps it as ValueError."""


def _word_char(ch: str) -> bool:
    return ch.isalnum() or ch == "_"


class _Scanner:
    def __init__(self, text: str) -> None:
        self.text = text
        self.pos = 0
        self.furthest = 0
        self.expected = []

    # -- primitives -----------------------------------------------------
    def _fail(self, what: str):
        if self.pos > self.furthest:
            self.furthest, self.expected = self.pos, [what]
        elif self.pos == self.furthest and what not in self.expected:
            self.expected.append(what)
        return None

    def ws(self) -> None:
        text, n = self.text, len(self.text)
        while self.pos < n and text[self.pos] in " \r\n\t":
            self.pos += 1

    def literal(self, token: str):
        if self.text.startswith(token, self.pos):
            self.pos += len(token)
            return token
        return self._fail(repr(token))

    def word(self):
        start, text, n = self.pos, self.text, len(self.text)
        while self.pos < n and _word_char(text[self.pos]):
            self.pos += 1
        if self.pos == start:
            return self._fail("letter or digit")
        return text[start:self.pos]

    def dashed_word(self):
        """``word ('-' word)*`` - mesh ids and annotation values."""
        start = self.pos
        if self.word() is None:
            return None
        while True:
            mark = self.pos
            if self.literal("-") is None or self.word() is None:
                self.pos = mark
                break
        return self.text[start:self.pos]

    # -- grammar rules ---------------------------------------------------
    def axis(self):
        name = self.word()
        if name is None:
            return None
        mark = self.pos
        self.ws()
        if self.literal("/") is not None:
            self.ws()
            mesh = self.dashed_word()
            if mesh is not None:
                return Axis(name, mesh)
        self.pos = mark
        return Axis(name)

    def group(self):
        if self.literal("(") is None:
            return None
        members = []
        while True:
            mark = self.pos
            self.ws()
            member = self.axis()
            if member is None:
                self.pos = mark
                break
            members.append(member)
        if not members:
            return None
        self.ws()
        if self.literal(")") is None:
            return None
        return AxisGroup(members)

    def axes(self):
        items = []
        while True:
            mark = self.pos
            self.ws()
            item = None
            for rule in (self.group, self.ellipsis, self.axis):
                inner = self.pos
                item = rule()
                if item is not None:
                    break
                self.pos = inner
            if item is None:
                self.pos = mark
                break
            items.append(item)
        return Axes(items) if items else None

    def ellipsis(self):
        return EllipsisAxis() if self.literal("...") is not None else None

    def partial(self):
        mark = self.pos
        self.ws()
        if self.literal("//") is None:
            self.pos = mark
            return None
        self.ws()
        inner = self.pos
        listed = self._partial_list()
        if listed is not None:
            return listed
        self.pos = inner
        mesh = self.dashed_word()
        if mesh is None:
            self.pos = mark
            return None
        return [mesh]

    def _partial_list(self):
        if self.literal("(") is None:
            return None
        self.ws()
        first = self.dashed_word()
        if first is None:
            return None
        names = [first]
        while True:
            mark = self.pos
            self.ws()
            if self.literal(",") is None:
                self.pos = mark
                break
            self.ws()
            name = self.dashed_word()
            if name is None:
                self.pos = mark
                break
            names.append(name)
        self.ws()
        if self.literal(")") is None:
            return None
        return names

    def annotation_value(self):
        start = self.pos
        if self.dashed_word() is None:
            return None
        mark = self.pos
        if self.literal(":") is None or self.word() is None:
            self.pos = mark
        return self.text[start:self.pos]

    def annotation_item(self):
        mark = self.pos
        if self.literal("param") is not None:
            return ("param", True)
        self.pos = mark
        for key in ("grad", "init_sync"):
            self.pos = mark
            if self.literal(key) is None:
                continue
            self.ws()
            if self.literal("=") is None:
                continue
            self.ws()
            value = self.annotation_value()
            if value is not None:
                return (key, value)
        self.pos = mark
        return None

    def annotation(self):
        mark = self.pos
        self.ws()
        if self.literal("[") is None:
            self.pos = mark
            return None
        self.ws()
        first = self.annotation_item()
        if first is None:
            self.pos = mark
            return None
        items = [first]
        while True:
            inner = self.pos
            self.ws()
            if self.literal(",") is None:
                self.pos = inner
                break
            self.ws()
            item = self.annotation_item()
            if item is None:
                self.pos = inner
                break
            items.append(item)
        self.ws()
        if self.literal("]") is None:
            self.pos = mark
            return None
        return TensorAnnotation.from_items(items)

    def tensor(self, allow_annotation: bool):
        axes = self.axes()
        if axes is None:
            return None
        partials = self.partial()
        annotation = self.annotation() if allow_annotation else None
        return TensorSpec(axes, partials or [], annotation)

    def expression(self):
        first = self.tensor(True)
        if first is None:
            raise self._error()
        self.ws()
        second = None
        mark = self.pos
        if self.literal(",") is not None:
            second = self.tensor(True)
            if second is None:
                self.pos = mark
            else:
                self.ws()
        if self.literal("->") is None:
            raise self._error()
        out = self.tensor(False)
        if out is None:
            raise self._error()
        if self.pos != len(self.text):
            self._fail("end of expression")
            raise self._error()
        return (first, second, out)

    def _error(self) -> EinshardSyntaxError:
        where = self.furthest
        found = self.text[where:where + 1] or "end of input"
        expected = " or ".join(self.expected) if self.expected else "more input"
        return EinshardSyntaxError(f"at character {where}: expected {expected}, found {found!r}")


class _RuleRunner:
    """``sharding(text).map()`` entry mirroring the reference grammar object."""

    def __init__(self, text: str) -> None:
        self._text = text

    def map(self):
        return _Scanner(self._text).expression()


def sharding(text: str) -> _RuleRunner:
    return _RuleRunner(text)


@lru_cache(maxsize=2048)
def _parse_cached(expression: str):
    return _Scanner(expression).expression()


def _clone_axis(axis):
    if isinstance(axis, AxisGroup):
        return AxisGroup(_clone_axis(member) for member in axis.axes)
    if isinstance(axis, EllipsisAxis):
        return EllipsisAxis()
    return Axis(axis.name, axis.shard_dim)


def _clone_spec(spec):
    if spec is None:
        return None
    return TensorSpec(Axes(_clone_axis(axis) for axis in spec.axes), spec.partials, spec.annotation)


def parse_sharding(expression: str):
    """Parse ``expression`` into ``(input0, input1 or None, output)`` specs.

    Any failure, syntactic or semantic, is reported as
    ``ValueError("Invalid einshard expression '<expr>': <detail>")``.
    """
    try:
        parsed = _parse_cached(expression)
    except Exception as error:  # noqa: BLE001 - uniform error surface
        raise ValueError(f"Invalid einshard expression {expression!r}: {error}") from error
    return tuple(_clone_spec(spec) for spec in parsed)
