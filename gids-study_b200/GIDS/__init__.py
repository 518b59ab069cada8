"""GIDS: GPU-initiated feature gather for GNN minibatches, B200 build.

Same import surface as the reference package (GIDS_Setup/GIDS/__init__.py:38,42).
"""
from .GIDS import GIDS, GIDS_DGLDataLoader  # noqa: F401
