"""``phew_b200.mx``: the ``mlx.core`` surface of phew's candidate path on B200.

Emitted ``output_source`` imports this module in place of ``mlx.core``; user
harness functions written against ``mx`` run on it unchanged.
"""

from . import fast  # noqa: F401
from .core import *  # noqa: F401,F403
from .extra import *  # noqa: F401,F403
from .extra import all, any, divmod, slice  # noqa: F401,A004  (MLX names)
from .core import (  # noqa: F401
    _elementwise,
    array,
    compile,
    eval,
    max,
    min,
    sum,
)
