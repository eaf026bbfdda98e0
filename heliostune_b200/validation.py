"""Exact-type checks used by the configuration dataclasses.

Behaviour follows ``src/heliostune/validation.py:12-120`` of the reference: ``bool`` is never
accepted where an ``int`` is expected, and every failure is a :class:`SchemaError`.
"""

from __future__ import annotations

import math
from collections.abc import Collection

from heliostune_b200.errors import SchemaError


def exact_object(value: object, *, context: str) -> dict[str, object]:
    if type(value) is not dict:
        raise SchemaError(f"{context} must be an object")
    if not all(type(key) is str for key in value):
        raise SchemaError(f"{context} object keys must be strings")
    return value


def exact_fields(value: object, *, required: Collection[str], context: str) -> dict[str, object]:
    data = exact_object(value, context=context)
    missing = sorted(set(required) - set(data))
    unknown = sorted(set(data) - set(required))
    problems = []
    if missing:
        problems.append(f"missing fields {missing!r}")
    if unknown:
        problems.append(f"unknown fields {unknown!r}")
    if problems:
        raise SchemaError(f"{context} has {' and '.join(problems)}")
    return data


def exact_bool(value: object, *, context: str) -> bool:
    if type(value) is not bool:
        raise SchemaError(f"{context} must be a boolean")
    return value


def exact_int(value: object, *, context: str, minimum: int | None = None) -> int:
    if type(value) is not int:
        raise SchemaError(f"{context} must be an integer")
    if minimum is not None and value < minimum:
        raise SchemaError(f"{context} must be at least {minimum}")
    return value


def finite_float(
    value: object,
    *,
    context: str,
    minimum: float | None = None,
    strictly_positive: bool = False,
) -> float:
    if type(value) not in (int, float):
        raise SchemaError(f"{context} must be a number")
    number = float(value)  # type: ignore[arg-type]
    if not math.isfinite(number):
        raise SchemaError(f"{context} must be finite")
    if strictly_positive and number <= 0:
        raise SchemaError(f"{context} must be positive")
    if minimum is not None and number < minimum:
        raise SchemaError(f"{context} must be at least {minimum}")
    return number


def nonblank_string(value: object, *, context: str) -> str:
    if type(value) is not str:
        raise SchemaError(f"{context} must be a string")
    if not value or value != value.strip():
        raise SchemaError(f"{context} must be nonblank with no surrounding whitespace")
    return value
