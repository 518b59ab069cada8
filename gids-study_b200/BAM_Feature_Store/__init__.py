"""BAM_Feature_Store: pybind11 module of the B200 GIDS feature store.

Drop-in for the reference package of the same name
(gids_module/BAM_Feature_Store/__init__.py:34, ``from .BAM_Feature_Store import *``).
The compiled module is built in-tree by ``python gids-study_b200/build.py``;
importing this package without it raises ImportError -- there is no CPU
fallback.
"""
from .BAM_Feature_Store import *  # noqa: F401,F403
from .BAM_Feature_Store import (  # noqa: F401
    BAM_Feature_Store_bfloat16,
    BAM_Feature_Store_float,
    BAM_Feature_Store_half,
    BAM_Feature_Store_long,
    GIDS_Controllers,
    version,
)
