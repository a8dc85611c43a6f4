"""Prototypes of the engine-level and remaining op-level entry points."""
from __future__ import annotations


def attach(lib, sig) -> None:  # extended as entry points are added
    return None
