"""Parallelism: flat buffers, data parallel bucket reduction, process meshes."""
from .flat import FlatParams  # noqa: F401
