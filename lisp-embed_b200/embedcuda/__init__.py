"""Host-side mirror of lisp-embed's embedding and IVF interfaces over
libembedcuda.so (sm_100a).

Modules follow the reference's packages: ``st`` (st.lisp), ``model``
(model.lisp), ``ann`` (ann.lisp) and ``kb`` (the scoring part of kb.lisp).
Token ids are the input; tokenisation stays with the caller.
"""
from . import _lib  # noqa: F401
from ._lib import EcError, init, shutdown  # noqa: F401
