"""GIDS: GPU-initiated feature gather for GNN minibatches, B200 build.

Same import surface as the reference package (GIDS_Setup/GIDS/__init__.py:38,42).
Importing the package (or ``GIDS.synthetic``) loads none of the compiled
libraries: the ``BAM_Feature_Store`` module is imported when the first ``GIDS``
object is constructed.
"""
from .GIDS import GIDS, GIDS_DGLDataLoader  # noqa: F401
