"""The two host bindings of the C ABI agree with its headers, argument by
argument: the ctypes table of the Python mirror (embedcuda/_lib.py) and the
sb-alien routines of the SBCL drop-in (lisp/cuda.lisp).  A binding that
passes an int where the header takes an int64_t (or a pointer where it takes
a size) corrupts its arguments without any error, so each parameter's kind
(pointer, signed / unsigned integer, float) and width are compared.  No GPU
and no SBCL are needed: the headers and the Lisp source are parsed as text."""
import ctypes as C
import os
import re

from embedcuda import _lib

REPO = _lib.REPO
HEADERS = [os.path.join(REPO, "include", "embedcuda.h"),
           os.path.join(REPO, "include", "embedcuda_debug.h")]
LISP = os.path.join(REPO, "lisp-embed_b200", "lisp", "cuda.lisp")

# scalar C types of the headers -> (kind, bytes)
C_SCALARS = {"int": ("i", 4), "int32_t": ("i", 4), "uint32_t": ("u", 4), "int64_t": ("i", 8),
             "long long": ("i", 8), "size_t": ("u", 8), "float": ("f", 4), "double": ("f", 8),
             "char": ("i", 1), "void": ("v", 0)}


def parse_headers():
    """{name: (return type, [parameter types])} with comments, preprocessor
    lines and parameter names removed; a type is ("ptr", pointee-type) or
    one of C_SCALARS' keys."""
    decls = {}
    for path in HEADERS:
        with open(path) as f:
            src = f.read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        src = re.sub(r"#[^\n]*", "", src)
        for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(ec[a-z]*_\w+)\s*\(([^)]*)\)\s*;", src):
            ret, name, args = m.group(1), m.group(2), m.group(3).strip()
            params = [] if args in ("", "void") else [_ctype(a, named=True) for a in args.split(",")]
            decls[name] = (_ctype(ret, named=False), params)
    return decls


def _ctype(text, named):
    t = " ".join(text.replace("*", " * ").split())
    words = t.split(" ")
    if named:  # drop the parameter name
        assert words[-1] != "*" and words[-1] not in C_SCALARS, text
        words = words[:-1]
    words = [w for w in words if w != "const"]
    stars = words.count("*")
    base = " ".join(w for w in words if w != "*")
    assert base in C_SCALARS, (text, base)
    if stars == 0:
        return base
    if stars == 1:
        return ("ptr", base)
    return ("ptr", ("ptr", base))


def _kind(t):
    return ("p", 8) if isinstance(t, tuple) else C_SCALARS[t]


# ---------------------------------------------------------------- ctypes --
def _ctypes_kind(ct):
    if ct is None:
        return ("v", 0)
    if ct in (C.c_void_p, C.c_char_p) or (isinstance(ct, type) and issubclass(ct, C._Pointer)):
        return ("p", 8)
    if ct in (C.c_float, C.c_double):
        return ("f", C.sizeof(ct))
    signed = ct(-1).value < 0
    return ("i" if signed else "u", C.sizeof(ct))


def _ctypes_pointee_ok(ct, c_type):
    """A typed ctypes pointer must point at the header's element type;
    c_void_p stands for any pointer, c_char_p only for char pointers."""
    if ct is C.c_void_p:
        return True
    pointee = c_type[1]
    if ct is C.c_char_p:
        return pointee == "char"
    target = ct._type_
    if isinstance(pointee, tuple):  # char *const * (an array of strings)
        return target is C.c_char_p and pointee == ("ptr", "char")
    if pointee == "void":
        return False
    return _ctypes_kind(target) == C_SCALARS[pointee]


def test_ctypes_table_matches_headers():
    decls = parse_headers()
    sigs = _lib._SIGS
    for name, (ret, args) in sigs.items():
        assert name in decls, f"{name}: bound but not declared"
        c_ret, c_params = decls[name]
        assert _ctypes_kind(ret) == _kind(c_ret), (name, "return", ret, c_ret)
        assert len(args) == len(c_params), (name, len(args), len(c_params))
        for i, (ct, c_t) in enumerate(zip(args, c_params)):
            assert _ctypes_kind(ct) == _kind(c_t), (name, i, ct, c_t)
            if isinstance(c_t, tuple):
                assert _ctypes_pointee_ok(ct, c_t), (name, i, ct, c_t)


def test_ctypes_table_covers_every_declaration():
    missing = sorted(set(parse_headers()) - set(_lib._SIGS))
    assert not missing, missing  # an unbound call would default every argument to int


# ------------------------------------------------------------------- Lisp --
def _read_sexps(src):
    """A small reader for the forms of cuda.lisp: lists, strings and atoms
    (comments dropped; reader macros such as #: and ' kept in the atom)."""
    toks = re.findall(r'"(?:\\.|[^"\\])*"|;[^\n]*|\(|\)|[^\s()";]+', src)
    stack, out = [[]], None
    for t in toks:
        if t.startswith(";"):
            continue
        if t == "(":
            stack.append([])
        elif t == ")":
            out = stack.pop()
            stack[-1].append(out)
        else:
            stack[-1].append(t)
    assert len(stack) == 1, "unbalanced parentheses"
    return stack[0]


LISP_SCALARS = {"sb-alien:int": ("i", 4), "sb-alien:unsigned-int": ("u", 4),
                "sb-alien:long": ("i", 8), "sb-alien:unsigned-long": ("u", 8),
                "sb-alien:single-float": ("f", 4), "sb-alien:double-float": ("f", 8),
                "sb-alien:void": ("v", 0)}


def _lisp_kind(t):
    if t in ("sb-sys:system-area-pointer", "sb-alien:c-string"):
        return ("p", 8)
    if isinstance(t, list) and len(t) == 2 and t[0] in ("sb-alien:signed", "sb-alien:unsigned"):
        return ("i" if t[0] == "sb-alien:signed" else "u", int(t[1]) // 8)
    return LISP_SCALARS[t]


def lisp_routines():
    with open(LISP) as f:
        forms = _read_sexps(f.read())
    out = {}
    for form in forms:
        if isinstance(form, list) and form and form[0] == "sb-alien:define-alien-routine":
            name = form[1][0].strip('"')
            out[name] = (form[2], [p[1] for p in form[3:]])
    return out


def test_lisp_routines_match_header():
    decls = parse_headers()
    routines = lisp_routines()
    assert {"ec_init", "ec_embed_batch", "ec_ann_build", "ec_ivf_search"} <= set(routines)
    for name, (ret, params) in routines.items():
        assert name in decls, f"{name}: bound in cuda.lisp but not declared"
        c_ret, c_params = decls[name]
        assert _lisp_kind(ret) == _kind(c_ret), (name, "return", ret, c_ret)
        if ret == "sb-alien:c-string":
            assert c_ret == ("ptr", "char"), name
        assert len(params) == len(c_params), (name, len(params), len(c_params))
        for i, (lt, c_t) in enumerate(zip(params, c_params)):
            assert _lisp_kind(lt) == _kind(c_t), (name, i, lt, c_t)
            if lt == "sb-alien:c-string":  # a Lisp string goes only where the header takes char *
                assert c_t == ("ptr", "char"), (name, i, c_t)


def _calls(form, heads, out):
    if isinstance(form, list):
        if form and isinstance(form[0], str) and form[0] in heads:
            out.append(form)
        for f in form:
            _calls(f, heads, out)
    return out


def test_lisp_call_sites_pass_every_parameter():
    """Each (%routine ...) call in cuda.lisp passes as many arguments as the
    routine declares (SBCL would only notice when compiling the file)."""
    with open(LISP) as f:
        forms = _read_sexps(f.read())
    arity = {}
    for form in forms:
        if isinstance(form, list) and form and form[0] == "sb-alien:define-alien-routine":
            arity[form[1][1]] = len(form) - 3
    calls = _calls([f for f in forms if not (isinstance(f, list) and f and
                                             f[0] == "sb-alien:define-alien-routine")], arity, [])
    called = {c[0] for c in calls}
    assert {"%init", "%embed-batch", "%kmeans", "%ann-build", "%ivf-search"} <= called, called
    for c in calls:
        assert len(c) - 1 == arity[c[0]], (c[0], len(c) - 1, arity[c[0]])


def test_reader_and_parser_catch_a_mismatch():
    """The comparisons above fail on a planted mismatch: an int where the
    header takes an int64_t, and a missing parameter."""
    decls = parse_headers()
    src = ('(sb-alien:define-alien-routine ("ec_kmeans" %k) sb-alien:int (x sb-sys:system-area-pointer) '
           '(n sb-alien:int))')
    (form,) = _read_sexps(src)
    params = [p[1] for p in form[3:]]
    c_params = decls["ec_kmeans"][1]
    assert _lisp_kind(params[1]) != _kind(c_params[1])
    assert len(params) != len(c_params)
    assert _ctypes_kind(C.c_int) != _kind("int64_t")
    assert not _ctypes_pointee_ok(C.POINTER(C.c_float), ("ptr", "int64_t"))
