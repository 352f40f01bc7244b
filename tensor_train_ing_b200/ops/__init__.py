"""sm_100a kernel library bindings and the autograd functions built on them."""
from ._ext import available, check_status, lib  # noqa: F401
