"""Host-side mirror of lisp-embed's embedding and IVF interfaces over
libembedcuda.so (sm_100a).

Modules follow the reference's packages: ``st`` (st.lisp), ``model``
(model.lisp), ``ann`` (ann.lisp), ``kb`` (the scoring part of kb.lisp) and
``tokenizer`` (tokenizer.lisp, through the library's ec_tokenize).  The
embedding calls take token ids; ``tokenizer`` turns texts into them.
"""
from . import _lib  # noqa: F401
from ._lib import EcError, init, shutdown  # noqa: F401
