"""Parser, spec data model, annotations and axis families."""

import pytest

import torch_einshard_b200 as es
from torch_einshard_b200.notation.parser import parse_sharding, sharding
from torch_einshard_b200.notation.families import cached_expand_axis_families, expand_family_mapping
from torch_einshard_b200.notation.spec import Axis, AxisGroup, EllipsisAxis, GradAnnotation, InitSyncAnnotation


def test_partials_single_and_list():
    x, y, z = sharding("b n h // tp -> b n h").map()
    assert y is None and x.partials == ("tp",) and z.partials == ()
    x, _, _ = sharding("loss // (sp1,sp2) -> loss").map()
    assert x.partials == ("sp1", "sp2")
    x, _, _ = sharding("loss // ( sp1-sp2 , dp-sp1-sp2 ) -> loss").map()
    assert x.partials == ("sp1-sp2", "dp-sp1-sp2")


def test_sharded_axes_groups_and_ellipsis():
    x, _, z = sharding("b n/tp h -> b n h // tp").map()
    assert x.axes[1] == Axis("n", "tp") and z.partials == ("tp",)
    x, _, z = sharding("b (h/sp p) c -> b h/sp p c").map()
    assert isinstance(x.axes[1], AxisGroup)
    assert [a.name for a in x.axes.flat()] == ["b", "h", "p", "c"]
    assert x.axes[1].axes[0].shard_dim == "sp"
    x, _, _ = sharding("... c -> ... c").map()
    assert isinstance(x.axes[0], EllipsisAxis)
    x, _, _ = sharding("a / tp-sp b -> a b").map()
    assert x.axes[0].shard_dim == "tp-sp"
    x, _, _ = sharding("a/sp_h b -> a b").map()
    assert x.axes[0].shard_dim == "sp_h"


def test_multiple_ellipsis_rejected():
    with pytest.raises(ValueError, match="at most one ellipsis"):
        sharding("... a ... -> a").map()


def test_annotations():
    x, y, z = parse_sharding("b c, out/tp c [param, grad=async] -> b out/tp")
    assert not x.annotation and y.annotation.is_param and not z.annotation
    assert y.annotation.grad == GradAnnotation(mode="inferred", backend="native", schedule="async")
    _, y, _ = parse_sharding("b c, out c [param, grad=dp:ddp] -> b out")
    assert y.annotation.grad.mesh_dims == ("dp",) and y.annotation.grad.backend == "ddp"
    _, y, _ = parse_sharding("b c, out c [param, grad=external, init_sync=none] -> b out")
    assert y.annotation.grad.backend == "external" and y.annotation.init_sync == InitSyncAnnotation(mode="none")
    _, y, _ = parse_sharding("b c, out c [param, grad = async] -> b out")
    assert y.annotation.grad.schedule == "async"


def test_repr_round_trip_and_cache_copies():
    expr = "b c, out/tp c [param, grad=sp1-sp2:async, init_sync=tp] -> b out/tp"
    first, second = parse_sharding(expr), parse_sharding(expr)
    assert first is not second and repr(first) == repr(second)
    assert repr(first[1]) == "out / tp × c [param, grad=sp1-sp2:async, init_sync=tp]"
    parsed = parse_sharding("a -> a")
    parsed[0].axes.append(Axis("b"))
    assert [a.name for a in parse_sharding("a -> a")[0].axes] == ["a"]


@pytest.mark.parametrize("bad", ["a b ->", "a -> a [param]", "a [async] -> a", "a -> a ", "-> a", "a, -> b",
                                 "a // -> a", "a [grad=] -> a", "(a -> a"])
def test_invalid_expressions(bad):
    with pytest.raises(ValueError, match="Invalid einshard expression"):
        parse_sharding(bad)
    with pytest.raises(ValueError, match="Invalid einshard expression"):
        es.einshard(bad) if bad != "-> a" else parse_sharding(bad)


def test_duplicate_annotation_and_bad_suffix():
    with pytest.raises(ValueError, match="Duplicate tensor annotation"):
        parse_sharding("a [param, param] -> a")
    with pytest.raises(ValueError, match="Unknown grad annotation suffix"):
        parse_sharding("a [grad=dp:bogus] -> a")
    with pytest.raises(ValueError, match="requires an explicit mesh group"):
        parse_sharding("a [grad=async:ddp] -> a")
    with pytest.raises(ValueError, match="do not accept suffixes"):
        parse_sharding("a [init_sync=dp:ddp] -> a")


def test_axis_families():
    expr = "b [*spatial *window] c -> b *spatial *window c"
    out, sizes = cached_expand_axis_families(expr, {"window": [4, 5]}, {"spatial": ["h", "w"], "window": ["wh", "ww"]})
    assert out == "b (h wh) (w ww) c -> b h w wh ww c" and sizes == {"wh": 4, "ww": 5}
    sizes["wh"] = 99
    _, again = cached_expand_axis_families(expr, {"window": [4, 5]}, {"spatial": ["h", "w"], "window": ["wh", "ww"]})
    assert again == {"wh": 4, "ww": 5}
    out, _ = cached_expand_axis_families("b [*s *w] c, o c [param, grad = async] -> b *s *w o", None,
                                         {"s": ("h", "w"), "w": ("wh", "ww")})
    assert out == "b (h wh) (w ww) c, o c [param, grad = async] -> b h w wh ww o"
    with pytest.raises(ValueError, match="matching lengths"):
        cached_expand_axis_families("[*a *b] -> x", None, {"a": ("p", "q"), "b": ("r",)})
    with pytest.raises(ValueError, match="Unknown axis family"):
        cached_expand_axis_families("*nope -> x", None, {"a": ("p",)})
    assert expand_family_mapping({"s": 2, "t": 1}, {"s": ("h", "w/sp")}, label="Shift") == {"h": 2, "w": 2, "t": 1}
    with pytest.raises(ValueError, match="has 1 values for 2 axes"):
        expand_family_mapping({"s": [1]}, {"s": ("h", "w")}, label="Halo")
