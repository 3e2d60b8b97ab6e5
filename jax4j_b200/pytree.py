"""PyTree / PyTrees (pytree/PyTree.java, pytree/PyTrees.java of the reference):
leaves, ordered lists and insertion-ordered maps of arrays."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List

from .core import IllegalArgumentException, NDArray


class PyTree:
    @staticmethod
    def leaf(value: NDArray) -> "Leaf":
        return Leaf(value)

    @staticmethod
    def list(*children: "PyTree") -> "ListNode":
        return ListNode(list(children))

    @staticmethod
    def dict(children: Dict[str, "PyTree"]) -> "MapNode":
        return MapNode(dict(children))

    @staticmethod
    def dictOf(arrays: Dict[str, NDArray]) -> "MapNode":
        return MapNode({k: Leaf(v) for k, v in arrays.items()})


@dataclass
class Leaf(PyTree):
    value: NDArray


@dataclass
class ListNode(PyTree):
    children: List[PyTree]


@dataclass
class MapNode(PyTree):
    children: Dict[str, PyTree]  # insertion-ordered


class PyTrees:
    @staticmethod
    def flatten(tree: PyTree) -> List[NDArray]:
        """PyTrees.flatten (PyTrees.java:25-35): depth-first, maps in insertion order."""
        out: List[NDArray] = []

        def rec(t):
            if isinstance(t, Leaf):
                out.append(t.value)
            elif isinstance(t, ListNode):
                for c in t.children:
                    rec(c)
            elif isinstance(t, MapNode):
                for c in t.children.values():
                    rec(c)
            else:
                raise IllegalArgumentException(f"not a PyTree: {type(t).__name__}")

        rec(tree)
        return out

    @staticmethod
    def unflatten(template: PyTree, leaves: List[NDArray]) -> PyTree:
        """PyTrees.unflatten (PyTrees.java:44-79)."""
        it = iter(leaves)

        def rec(t):
            if isinstance(t, Leaf):
                try:
                    return Leaf(next(it))
                except StopIteration:
                    raise IllegalArgumentException("Not enough leaves for this tree structure") from None
            if isinstance(t, ListNode):
                return ListNode([rec(c) for c in t.children])
            return MapNode({k: rec(v) for k, v in t.children.items()})

        result = rec(template)
        if next(it, None) is not None:
            raise IllegalArgumentException("Too many leaves for this tree structure")
        return result

    @staticmethod
    def map(fn: Callable[[NDArray], NDArray], tree: PyTree) -> PyTree:
        """PyTrees.map (PyTrees.java:80-91)."""
        return PyTrees.unflatten(tree, [fn(x) for x in PyTrees.flatten(tree)])

    @staticmethod
    def map2(fn: Callable[[NDArray, NDArray], NDArray], a: PyTree, b: PyTree) -> PyTree:
        """PyTrees.map2 (PyTrees.java:97-105)."""
        al, bl = PyTrees.flatten(a), PyTrees.flatten(b)
        if len(al) != len(bl):
            raise IllegalArgumentException(
                f"Tree structures do not match: {len(al)} vs {len(bl)} leaves")
        return PyTrees.unflatten(a, [fn(x, y) for x, y in zip(al, bl)])
