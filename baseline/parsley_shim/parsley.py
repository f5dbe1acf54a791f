"""Minimal stand-in for the ``parsley`` package, used only by ``bench.py --impl reference``.

The reference implementation depends on parsley (a PEG parser generator) for
its expression grammar; parsley is not installable offline here.  This module
provides ``makeGrammar(source, bindings, name)`` for that one grammar: the
returned object parses expressions with a hand-written recursive-descent
scanner and builds the objects with the classes found in ``bindings`` (the
reference's own ``Axis``, ``Axes``, ``AxisGroup``, ``EllipsisAxis``,
``TensorAnnotation`` and ``TensorSpec``).  Everything after parsing - planner,
executor, collectives and einsum - is the unmodified reference code.
"""

__all__ = ["makeGrammar", "ParseError"]


class ParseError(Exception):
    pass


def _word_char(ch):
    return ch.isalnum() or ch == "_"


class _Scanner:
    def __init__(self, text, b):
        self.t, self.p, self.b = text, 0, b

    def ws(self):
        while self.p < len(self.t) and self.t[self.p] in " \r\n\t":
            self.p += 1

    def lit(self, s):
        if self.t.startswith(s, self.p):
            self.p += len(s)
            return True
        return False

    def word(self):
        q = self.p
        while self.p < len(self.t) and _word_char(self.t[self.p]):
            self.p += 1
        return self.t[q:self.p] if self.p > q else None

    def dashed(self):
        q = self.p
        if self.word() is None:
            return None
        while True:
            m = self.p
            if not (self.lit("-") and self.word() is not None):
                self.p = m
                break
        return self.t[q:self.p]

    def axis(self):
        name = self.word()
        if name is None:
            return None
        m = self.p
        self.ws()
        if self.lit("/"):
            self.ws()
            mesh = self.dashed()
            if mesh is not None:
                return self.b["Axis"](name, mesh)
        self.p = m
        return self.b["Axis"](name)

    def group(self):
        if not self.lit("("):
            return None
        members = []
        while True:
            m = self.p
            self.ws()
            a = self.axis()
            if a is None:
                self.p = m
                break
            members.append(a)
        self.ws()
        if not members or not self.lit(")"):
            return None
        return self.b["AxisGroup"](members)

    def axes(self):
        items = []
        while True:
            m = self.p
            self.ws()
            item = None
            for rule in (self.group, lambda: self.b["EllipsisAxis"]() if self.lit("...") else None, self.axis):
                q = self.p
                item = rule()
                if item is not None:
                    break
                self.p = q
            if item is None:
                self.p = m
                break
            items.append(item)
        return self.b["Axes"](items) if items else None

    def partial(self):
        m = self.p
        self.ws()
        if not self.lit("//"):
            self.p = m
            return None
        self.ws()
        q = self.p
        if self.lit("("):
            self.ws()
            first = self.dashed()
            if first is not None:
                names = [first]
                while True:
                    r = self.p
                    self.ws()
                    if not self.lit(","):
                        self.p = r
                        break
                    self.ws()
                    nxt = self.dashed()
                    if nxt is None:
                        self.p = r
                        break
                    names.append(nxt)
                self.ws()
                if self.lit(")"):
                    return names
        self.p = q
        mesh = self.dashed()
        if mesh is None:
            self.p = m
            return None
        return [mesh]

    def value(self):
        q = self.p
        if self.dashed() is None:
            return None
        m = self.p
        if not (self.lit(":") and self.word() is not None):
            self.p = m
        return self.t[q:self.p]

    def item(self):
        m = self.p
        if self.lit("param"):
            return ("param", True)
        for key in ("grad", "init_sync"):
            self.p = m
            if self.lit(key):
                self.ws()
                if self.lit("="):
                    self.ws()
                    v = self.value()
                    if v is not None:
                        return (key, v)
        self.p = m
        return None

    def annotation(self):
        m = self.p
        self.ws()
        if not self.lit("["):
            self.p = m
            return None
        self.ws()
        first = self.item()
        if first is None:
            self.p = m
            return None
        items = [first]
        while True:
            q = self.p
            self.ws()
            if not self.lit(","):
                self.p = q
                break
            self.ws()
            it = self.item()
            if it is None:
                self.p = q
                break
            items.append(it)
        self.ws()
        if not self.lit("]"):
            self.p = m
            return None
        return self.b["TensorAnnotation"].from_items(items)

    def tensor(self, annotated):
        axes = self.axes()
        if axes is None:
            return None
        partials = self.partial()
        ann = self.annotation() if annotated else None
        return self.b["TensorSpec"](axes, partials or [], ann) if annotated else self.b["TensorSpec"](axes, partials or [])

    def map(self):
        first = self.tensor(True)
        if first is None:
            raise ParseError(f"cannot parse {self.t!r}")
        self.ws()
        second = None
        m = self.p
        if self.lit(","):
            second = self.tensor(True)
            if second is None:
                self.p = m
            else:
                self.ws()
        if not self.lit("->"):
            raise ParseError(f"expected '->' at {self.p} in {self.t!r}")
        out = self.tensor(False)
        if out is None or self.p != len(self.t):
            raise ParseError(f"expected EOF at {self.p} in {self.t!r}")
        return (first, second, out)


def makeGrammar(source, bindings, name="Grammar"):
    class _Grammar:
        def __init__(self, text):
            self._text = text

        def map(self):
            return _Scanner(self._text, bindings).map()

    _Grammar.__name__ = name
    return _Grammar
