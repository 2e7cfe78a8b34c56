"""Alias package, as in the reference (mlx_mhc/__init__.py re-exports mhc_mlx)."""

from mhc_mlx import *  # noqa: F401,F403
from mhc_mlx import __version__  # noqa: F401
