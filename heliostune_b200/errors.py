"""Failure types of the heliostune_b200 host layer.

The hierarchy mirrors the reference's ``heliostune.errors`` (``src/heliostune/errors.py:6-19``)
so callers that catch ``HeliostuneError``, ``SchemaError`` or ``ProtocolError`` keep working:
schema and protocol failures are also ``ValueError``.
"""

from __future__ import annotations


class HeliostuneError(Exception):
    """Base class for failures that are safe to show to a user."""


class SchemaError(HeliostuneError, ValueError):
    """A value does not satisfy a configuration or record schema."""


class ArtifactError(HeliostuneError):
    """An artifact could not be read or written safely."""


class ProtocolError(HeliostuneError, ValueError):
    """A request violates a frozen measurement or collection protocol."""


class KernelError(HeliostuneError, RuntimeError):
    """The native library reported a launch failure or a device-side timeout."""
