"""Runs the reference's own TypeScript source on the CPU, with JavaScript's
number semantics, to produce golden vectors for the oracle.

There is no JavaScript runtime in this image, so this module translates the
TypeScript subset that the reference's CPU path is written in into Python
and executes it. It is test infrastructure: only the fixture generator
beside it imports it, and nothing under krystal_b200/ or oracle/ does.

What it preserves, because parity depends on it:
* every number is an IEEE double (Python float, or an exact Python int while
  a value is integral; `/` of two integers that divides exactly stays an int
  so it can index an array, which is the same double);
* `Float32Array` element stores round to f32 (round to nearest even: the
  arrays are `array.array('f')`), reads widen exactly; `Uint32Array` and the
  other integer arrays wrap stores with ToUint32 / ToInt32 / ...;
* `| & ^ ~ << >> >>>` and `Math.imul` use ToInt32 / ToUint32;
* `%` has the sign of the dividend; `Math.max`/`min` propagate NaN;
  `Math.exp` overflows to Infinity; `Math.log` of 0 / negatives gives
  -Infinity / NaN;
* loop orders, evaluation order of `+=` chains and the f32 store points are
  the source's own, since the source is what runs.

Known limits (none met by the files it is used on, and each one fails
loudly rather than silently where it can): NaN counts as true in a
condition; a negative array index wraps instead of reading undefined; a
`subarray` of an owned typed array is a copy that refuses writes (views
made over an ArrayBuffer do alias it); closures
capture loop variables by reference; labels, generators and
regular-expression literals are not translated. `Math.exp/log/sin/cos` are
the C library's (as the C++ oracle's), which may differ from V8's in the
last bit in rare cases.
"""
from __future__ import annotations

import array
import functools
import keyword
import math
import re
import struct
import sys
from pathlib import Path

# ---------------------------------------------------------------------------
# tokenizer
# ---------------------------------------------------------------------------

PUNCS = sorted(""">>>= ... === !== **= <<= >>= >>> &&= ||= ??= => == != <= >= && || ?? ?. ++ -- += -= *= /= %= &= |= ^=
<< >> ** { } ( ) [ ] ; , < > + - * / % & | ^ ! ~ ? : = . @ #""".split(), key=len, reverse=True)
NUM_RE = re.compile(r"(?:0[xX][0-9a-fA-F_]+|0[bB][01_]+|0[oO][0-7_]+|(?:\d[\d_]*(?:\.[\d_]*)?|\.\d[\d_]*)(?:[eE][+-]?\d[\d_]*)?)n?")
IDENT_RE = re.compile(r"[A-Za-z_$][A-Za-z0-9_$]*")


class Tok:
    __slots__ = ("kind", "value", "pos", "nl")

    def __init__(self, kind, value, pos, nl):
        self.kind, self.value, self.pos, self.nl = kind, value, pos, nl

    def __repr__(self):
        return f"Tok({self.kind},{self.value!r})"


def _read_string(src, i):
    q = src[i]
    out = []
    i += 1
    while src[i] != q:
        c = src[i]
        if c == "\\":
            i += 1
            c = src[i]
            if c == "n":
                out.append("\n")
            elif c == "t":
                out.append("\t")
            elif c == "r":
                out.append("\r")
            elif c == "0":
                out.append("\0")
            elif c == "u":
                if src[i + 1] == "{":
                    j = src.index("}", i)
                    out.append(chr(int(src[i + 2:j], 16)))
                    i = j
                else:
                    out.append(chr(int(src[i + 1:i + 5], 16)))
                    i += 4
            elif c == "x":
                out.append(chr(int(src[i + 1:i + 3], 16)))
                i += 2
            elif c == "\n":
                pass
            else:
                out.append(c)
        else:
            out.append(c)
        i += 1
    return "".join(out), i + 1


def _read_template(src, i):
    """-> ([str parts], [expression source texts]), index after the closing backtick."""
    i += 1
    strs, exprs, cur = [], [], []
    while True:
        c = src[i]
        if c == "`":
            strs.append("".join(cur))
            return (strs, exprs), i + 1
        if c == "\\":
            if src[i + 1] == "u":
                s, _ = _read_string('"' + src[i:i + 6] + '"', 0)
                i += 6
            else:
                s, _ = _read_string('"' + src[i:i + 2] + '"', 0)
                i += 2
            cur.append(s)
            continue
        if c == "$" and src[i + 1] == "{":
            strs.append("".join(cur))
            cur = []
            depth, j = 1, i + 2
            while depth:
                ch = src[j]
                if ch in "\"'":
                    _, j = _read_string(src, j)
                    continue
                if ch == "`":
                    _, j = _read_template(src, j)
                    continue
                if ch == "{":
                    depth += 1
                elif ch == "}":
                    depth -= 1
                j += 1
            exprs.append(src[i + 2:j - 1])
            i = j
            continue
        cur.append(c)
        i += 1


def tokenize(src):
    toks = []
    i, n, nl = 0, len(src), False
    while i < n:
        c = src[i]
        if c in " \t\r﻿":
            i += 1
            continue
        if c == "\n":
            nl = True
            i += 1
            continue
        if src.startswith("//", i):
            j = src.find("\n", i)
            i = n if j < 0 else j
            continue
        if src.startswith("/*", i):
            j = src.index("*/", i + 2)
            nl = nl or "\n" in src[i:j]
            i = j + 2
            continue
        if c.isdigit() or (c == "." and i + 1 < n and src[i + 1].isdigit()):
            m = NUM_RE.match(src, i)
            s = m.group(0).replace("_", "")
            if s.endswith("n"):
                raise SyntaxError("BigInt literals are not supported")
            if s[:2] in ("0x", "0X"):
                v = int(s[2:], 16)
            elif s[:2] in ("0b", "0B"):
                v = int(s[2:], 2)
            elif s[:2] in ("0o", "0O"):
                v = int(s[2:], 8)
            elif any(ch in s for ch in ".eE"):
                v = float(s)
                if v.is_integer() and abs(v) < 2 ** 53 and "e" not in s.lower():
                    v = int(v)
            else:
                v = int(s)
            toks.append(Tok("num", v, i, nl))
            i = m.end()
            nl = False
            continue
        if c.isalpha() or c in "_$":
            m = IDENT_RE.match(src, i)
            toks.append(Tok("name", m.group(0), i, nl))
            i = m.end()
            nl = False
            continue
        if c in "\"'":
            s, j = _read_string(src, i)
            toks.append(Tok("str", s, i, nl))
            i, nl = j, False
            continue
        if c == "`":
            t, j = _read_template(src, i)
            toks.append(Tok("tmpl", t, i, nl))
            i, nl = j, False
            continue
        for p in PUNCS:
            if src.startswith(p, i):
                if p == "?." and i + 2 < n and src[i + 2].isdigit():
                    continue
                toks.append(Tok("punc", p, i, nl))
                i += len(p)
                nl = False
                break
        else:
            raise SyntaxError(f"unexpected character {c!r} at {i}")
    toks.append(Tok("eof", None, n, True))
    return toks


# ---------------------------------------------------------------------------
# parser: TypeScript -> a small AST of tuples; types are skipped
# ---------------------------------------------------------------------------

ASSIGN_OPS = {"=", "+=", "-=", "*=", "/=", "%=", "**=", "<<=", ">>=", ">>>=", "&=", "|=", "^=", "&&=", "||=", "??="}
BINPREC = {"??": 1, "||": 2, "&&": 3, "|": 4, "^": 5, "&": 6, "==": 7, "!=": 7, "===": 7, "!==": 7,
           "<": 8, ">": 8, "<=": 8, ">=": 8, "instanceof": 8, "in": 8, "<<": 9, ">>": 9, ">>>": 9,
           "+": 10, "-": 10, "*": 11, "/": 11, "%": 11, "**": 12}
MODIFIERS = {"public", "private", "protected", "readonly", "static", "abstract", "override", "declare", "accessor"}


class Parser:
    def __init__(self, src, fname="<ts>"):
        self.toks = tokenize(src)
        self.i = 0
        self.fname = fname
        self.src = src

    # -- token helpers
    @property
    def tok(self):
        return self.toks[self.i]

    def peek(self, k=1):
        return self.toks[min(self.i + k, len(self.toks) - 1)]

    def at(self, v):
        t = self.tok
        return t.kind == "punc" and t.value == v

    def at_name(self, v=None):
        t = self.tok
        return t.kind == "name" and (v is None or t.value == v)

    def next(self):
        t = self.toks[self.i]
        self.i += 1
        return t

    def expect(self, v):
        if not self.at(v):
            self.error(f"expected {v!r}")
        return self.next()

    def error(self, msg):
        t = self.tok
        line = self.src.count("\n", 0, t.pos) + 1
        raise SyntaxError(f"{self.fname}:{line}: {msg}, got {t.kind} {t.value!r}")

    def name(self):
        t = self.tok
        if t.kind != "name":
            self.error("expected a name")
        self.i += 1
        return t.value

    def semi(self):
        if self.at(";"):
            self.next()

    # -- types (skipped)
    def skip_balanced(self):
        pairs = {"(": ")", "[": "]", "{": "}"}
        depth = 0
        while True:
            t = self.next()
            if t.kind == "eof":
                self.error("unbalanced brackets")
            if t.kind == "punc":
                if t.value in pairs:
                    depth += 1
                elif t.value in (")", "]", "}"):
                    depth -= 1
            if depth == 0:
                return

    def skip_angle(self):
        self.expect("<")
        depth = 1
        while depth > 0:
            t = self.tok
            if t.kind == "eof":
                self.error("unbalanced <")
            if t.kind == "punc":
                if t.value == "<":
                    depth += 1
                elif t.value == ">":
                    depth -= 1
                elif t.value == ">>":
                    depth -= 2
                elif t.value == ">>>":
                    depth -= 3
                elif t.value in ("(", "[", "{"):
                    self.skip_balanced()
                    continue
                elif t.value == ">=":
                    depth -= 1
                    t.value = "="
                    if depth == 0:
                        return
                    continue
            self.next()
        if depth < 0:
            self.error("split >> in a type")

    def skip_type(self):
        if self.at("|") or self.at("&"):
            self.next()
        self.skip_postfix_type()
        while self.at("|") or self.at("&"):
            self.next()
            self.skip_postfix_type()
        if self.at_name("extends"):  # conditional type
            self.next()
            self.skip_type()
            self.expect("?")
            self.skip_type()
            self.expect(":")
            self.skip_type()

    def skip_postfix_type(self):
        self.skip_primary_type()
        while self.at("[") and not self.tok.nl:
            self.skip_balanced()

    def skip_primary_type(self):
        t = self.tok
        if t.kind == "name" and t.value in ("readonly", "keyof", "unique", "infer", "asserts"):
            self.next()
            return self.skip_postfix_type()
        if t.kind == "name" and t.value == "typeof":
            self.next()
            self.name()
            while self.at("."):
                self.next()
                self.name()
            return
        if t.kind == "name" and t.value == "new":
            self.next()
            return self.skip_primary_type()
        if self.at("<"):
            self.skip_angle()
            return self.skip_primary_type()
        if self.at("("):
            self.skip_balanced()
            if self.at("=>"):
                self.next()
                self.skip_type()
            return
        if self.at("{") or self.at("["):
            self.skip_balanced()
            return
        if self.at("-"):
            self.next()
        if t.kind in ("str", "num", "tmpl"):
            self.next()
            return
        self.name()
        while self.at("."):
            self.next()
            self.name()
        if self.at("<") and not self.tok.nl:
            self.skip_angle()
        if self.at_name("is"):
            self.next()
            self.skip_type()

    # -- program
    def program(self):
        body = []
        while self.tok.kind != "eof":
            s = self.statement()
            if s is not None:
                body.append(s)
        return body

    def statement(self):
        t = self.tok
        if t.kind == "punc":
            if t.value == "{":
                return ("block", self.block())
            if t.value == ";":
                self.next()
                return None
            if t.value == "@":
                self.error("decorators are not supported")
        if t.kind == "name":
            v = t.value
            nxt = self.peek()
            if v in ("const", "let", "var") and (nxt.kind == "name" or (nxt.kind == "punc" and nxt.value in ("{", "["))):
                if v == "const" and nxt.kind == "name" and nxt.value == "enum":
                    self.next()
                    return self.enum_decl()
                d = self.var_decl()
                self.semi()
                return d
            if v == "function" or (v == "async" and nxt.kind == "name" and nxt.value == "function" and not nxt.nl):
                return self.function_decl()
            if v == "class" or (v == "abstract" and nxt.kind == "name" and nxt.value == "class"):
                if v == "abstract":
                    self.next()
                return self.class_decl()
            if v == "interface" and nxt.kind == "name":
                self.next()
                self.name()
                if self.at("<"):
                    self.skip_angle()
                while not self.at("{"):
                    self.next()
                self.skip_balanced()
                return None
            if v == "type" and nxt.kind == "name" and not nxt.nl:
                self.next()
                self.name()
                if self.at("<"):
                    self.skip_angle()
                self.expect("=")
                self.skip_type()
                self.semi()
                return None
            if v == "declare" and nxt.kind == "name" and not nxt.nl:
                self.next()
                if self.at_name("global") or self.at_name("module") or self.at_name("namespace"):
                    self.next()
                    if self.tok.kind == "str" or self.at_name():
                        self.next()
                    self.skip_balanced()
                    return None
                while not self.at(";") and not self.tok.nl:
                    if self.at("{") or self.at("(") or self.at("["):
                        self.skip_balanced()
                    else:
                        self.next()
                self.semi()
                return None
            if v == "enum":
                return self.enum_decl()
            if v == "import" and not (nxt.kind == "punc" and nxt.value in ("(", ".")):
                return self.import_decl()
            if v == "export":
                return self.export_decl()
            if v == "return":
                self.next()
                e = None
                if not (self.at(";") or self.at("}") or self.tok.nl or self.tok.kind == "eof"):
                    e = self.expr()
                self.semi()
                return ("ret", e)
            if v == "if":
                self.next()
                self.expect("(")
                c = self.expr()
                self.expect(")")
                a = self.statement()
                b = None
                if self.at_name("else"):
                    self.next()
                    b = self.statement()
                return ("if", c, a, b)
            if v == "for":
                return self.for_stmt()
            if v == "while":
                self.next()
                self.expect("(")
                c = self.expr()
                self.expect(")")
                return ("while", c, self.statement())
            if v == "do":
                self.next()
                body = self.statement()
                if not self.at_name("while"):
                    self.error("expected while")
                self.next()
                self.expect("(")
                c = self.expr()
                self.expect(")")
                self.semi()
                return ("dowhile", body, c)
            if v in ("break", "continue"):
                self.next()
                if self.at_name() and not self.tok.nl:
                    self.error("labels are not supported")
                self.semi()
                return (v,)
            if v == "throw":
                self.next()
                e = self.expr()
                self.semi()
                return ("throw", e)
            if v == "try":
                self.next()
                blk = self.block()
                param, handler, fin = None, None, None
                if self.at_name("catch"):
                    self.next()
                    if self.at("("):
                        self.next()
                        param = self.binding()
                        if self.at(":"):
                            self.next()
                            self.skip_type()
                        self.expect(")")
                    handler = self.block()
                if self.at_name("finally"):
                    self.next()
                    fin = self.block()
                return ("try", blk, param, handler, fin)
            if v == "switch":
                return self.switch_stmt()
            if nxt.kind == "punc" and nxt.value == ":" and v not in ("default", "case"):
                self.error("labels are not supported")
        e = self.expr()
        self.semi()
        return ("expr", e)

    def block(self):
        self.expect("{")
        body = []
        while not self.at("}"):
            s = self.statement()
            if s is not None:
                body.append(s)
        self.next()
        return body

    def enum_decl(self):
        self.next()
        name = self.name()
        self.expect("{")
        members, cur = [], -1
        while not self.at("}"):
            key = self.next().value
            if self.at("="):
                self.next()
                val = self.assign()
            else:
                val = ("num", cur + 1)
            cur = val[1] if val[0] == "num" else cur + 1
            members.append((key, val))
            if self.at(","):
                self.next()
        self.next()
        return ("var", "const", [(("id", name), ("obj", [("kv", k, v) for k, v in members]))])

    def var_decl(self):
        kind = self.next().value
        decls = []
        while True:
            pat = self.binding()
            if self.at("!"):
                self.next()
            if self.at(":"):
                self.next()
                self.skip_type()
            init = None
            if self.at("="):
                self.next()
                init = self.assign()
            decls.append((pat, init))
            if self.at(","):
                self.next()
                continue
            break
        return ("var", kind, decls)

    def binding(self):
        """A binding pattern: ('id', n) | ('opat', [(key, pat, default)], rest) | ('apat', [(pat, default)|None], rest)."""
        if self.at("{"):
            self.next()
            props, rest = [], None
            while not self.at("}"):
                if self.at("..."):
                    self.next()
                    rest = self.binding()
                else:
                    t = self.next()
                    if t.kind == "punc" and t.value == "[":
                        self.error("computed keys in patterns are not supported")
                    key = t.value
                    if self.at(":"):
                        self.next()
                        pat = self.binding()
                    else:
                        pat = ("id", key)
                    dflt = None
                    if self.at("="):
                        self.next()
                        dflt = self.assign()
                    props.append((str(key), pat, dflt))
                if self.at(","):
                    self.next()
            self.next()
            return ("opat", props, rest)
        if self.at("["):
            self.next()
            elems, rest = [], None
            while not self.at("]"):
                if self.at(","):
                    self.next()
                    elems.append(None)
                    continue
                if self.at("..."):
                    self.next()
                    rest = self.binding()
                else:
                    pat = self.binding()
                    dflt = None
                    if self.at("="):
                        self.next()
                        dflt = self.assign()
                    elems.append((pat, dflt))
                if self.at(","):
                    self.next()
            self.next()
            return ("apat", elems, rest)
        return ("id", self.name())

    def params(self):
        """'(' params ')' -> [(pattern, default, is_rest, field_name_or_None)]"""
        self.expect("(")
        out = []
        while not self.at(")"):
            field = False
            while self.at_name() and self.tok.value in MODIFIERS and self.peek().kind == "name":
                self.next()
                field = True
            rest = False
            if self.at("..."):
                self.next()
                rest = True
            if self.at_name("this") and self.peek().kind == "punc" and self.peek().value == ":":
                self.next()
                self.next()
                self.skip_type()
                if self.at(","):
                    self.next()
                continue
            pat = self.binding()
            if self.at("?"):
                self.next()
            if self.at(":"):
                self.next()
                self.skip_type()
            dflt = None
            if self.at("="):
                self.next()
                dflt = self.assign()
            out.append((pat, dflt, rest, pat[1] if field else None))
            if self.at(","):
                self.next()
        self.next()
        return out

    def function_rest(self, name):
        if self.at("<"):
            self.skip_angle()
        params = self.params()
        if self.at(":"):
            self.next()
            self.skip_type()
        if not self.at("{"):  # an overload signature
            self.semi()
            return None
        body = self.block()
        return ("fn", params, body, False, False, name)

    def function_decl(self):
        if self.at_name("async"):
            self.next()
        self.next()  # function
        if self.at("*"):
            self.error("generators are not supported")
        name = self.name()
        f = self.function_rest(name)
        if f is None:
            return None
        return ("fundecl", name, f)

    def class_decl(self, expr=False):
        self.next()  # class
        name = self.name() if self.at_name() and not self.at_name("extends") and not self.at_name("implements") else None
        if self.at("<"):
            self.skip_angle()
        sup = None
        if self.at_name("extends"):
            self.next()
            sup = self.call_member(no_call=False)
            if self.at("<"):
                self.skip_angle()
        if self.at_name("implements"):
            self.next()
            while not self.at("{"):
                self.next()
        self.expect("{")
        members = []
        while not self.at("}"):
            if self.at(";"):
                self.next()
                continue
            static = False
            while self.at_name() and self.tok.value in MODIFIERS and not (
                    self.peek().kind == "punc" and self.peek().value in ("(", "=", ";", ":", "?", "!", "<")):
                if self.tok.value == "static":
                    static = True
                self.next()
            kind = "method"
            if self.at_name("get") or self.at_name("set"):
                p = self.peek()
                if p.kind == "name" or (p.kind == "punc" and p.value in ("[", "#")) or p.kind == "str":
                    kind = self.next().value
            if self.at_name("async") and self.peek().kind == "name":
                self.next()
            if self.at("#"):
                self.next()
                mname = "_p_" + self.name()
            elif self.at("["):
                self.error("computed class members are not supported")
            else:
                mname = self.next().value
            if self.at("?") or self.at("!"):
                self.next()
            if self.at("(") or self.at("<"):
                f = self.function_rest(mname)
                if f is not None:
                    members.append((kind if mname != "constructor" else "ctor", mname, f, static))
                continue
            if self.at(":"):
                self.next()
                self.skip_type()
            init = None
            if self.at("="):
                self.next()
                init = self.assign()
            self.semi()
            members.append(("field", mname, init, static))
        self.next()
        node = ("class", name, sup, members)
        return node if expr else ("classdecl", name, node)

    def import_decl(self):
        self.next()
        if self.at_name("type") and not (self.peek().kind == "punc" and self.peek().value == ",") \
                and not (self.peek().kind == "name" and self.peek().value == "from"):
            while self.tok.kind != "str":
                self.next()
            self.next()
            self.semi()
            return None
        names, default, star = [], None, None
        if self.tok.kind == "str":
            spec = self.next().value
            self.semi()
            return ("import", spec, [], None, None)
        if self.at_name() and not self.at_name("from"):
            default = self.name()
            if self.at(","):
                self.next()
        if self.at("*"):
            self.next()
            if not self.at_name("as"):
                self.error("expected as")
            self.next()
            star = self.name()
        if self.at("{"):
            self.next()
            while not self.at("}"):
                is_type = False
                if self.at_name("type") and self.peek().kind == "name" and self.peek().value != "as":
                    self.next()
                    is_type = True
                n = self.next().value
                alias = n
                if self.at_name("as"):
                    self.next()
                    alias = self.next().value
                if not is_type:
                    names.append((n, alias))
                if self.at(","):
                    self.next()
            self.next()
        if not self.at_name("from"):
            self.error("expected from")
        self.next()
        spec = self.next().value
        if self.at_name("with") or self.at_name("assert"):
            self.next()
            self.skip_balanced()
        self.semi()
        return ("import", spec, names, default, star)

    def export_decl(self):
        self.next()
        if self.at_name("default"):
            self.next()
            if self.at_name("function") or self.at_name("class"):
                s = self.statement()
                return ("block_seq", [s, ("expr", ("asg", "=", ("id", "__default__"), ("id", s[1])))])
            e = self.assign()
            self.semi()
            return ("var", "const", [(("id", "__default__"), e)])
        if self.at_name("type") and self.peek().kind == "punc" and self.peek().value == "{":
            self.next()
            self.skip_balanced()
            if self.at_name("from"):
                self.next()
                self.next()
            self.semi()
            return None
        if self.at("*"):
            self.next()
            alias = None
            if self.at_name("as"):
                self.next()
                alias = self.name()
            self.next()  # from
            spec = self.next().value
            self.semi()
            return ("import", spec, [], None, alias) if alias else ("exportstar", spec)
        if self.at("{"):
            self.next()
            names = []
            while not self.at("}"):
                if self.at_name("type") and self.peek().kind == "name":
                    self.next()
                    self.next()
                    if self.at_name("as"):
                        self.next()
                        self.next()
                else:
                    n = self.next().value
                    alias = n
                    if self.at_name("as"):
                        self.next()
                        alias = self.next().value
                    names.append((n, alias))
                if self.at(","):
                    self.next()
            self.next()
            if self.at_name("from"):
                self.next()
                spec = self.next().value
                self.semi()
                return ("import", spec, names, None, None)
            self.semi()
            return ("exportnames", names)
        return self.statement()

    def for_stmt(self):
        self.next()
        if self.at_name("await"):
            self.error("for await is not supported")
        self.expect("(")
        init = None
        if self.at_name() and self.tok.value in ("const", "let", "var"):
            save = self.i
            kind = self.next().value
            pat = self.binding()
            if self.at_name("of") or self.at_name("in"):
                which = self.next().value
                it = self.assign() if which == "of" else self.expr()
                self.expect(")")
                return ("forof" if which == "of" else "forin", kind, pat, it, self.statement())
            self.i = save
            init = self.var_decl()
        elif not self.at(";"):
            save = self.i
            e = self.call_member()
            if self.at_name("of"):
                self.next()
                it = self.assign()
                self.expect(")")
                return ("forof", None, e, it, self.statement())
            self.i = save
            init = ("expr", self.expr())
        self.expect(";")
        test = None if self.at(";") else self.expr()
        self.expect(";")
        update = None if self.at(")") else self.expr()
        self.expect(")")
        return ("for", init, test, update, self.statement())

    def switch_stmt(self):
        self.next()
        self.expect("(")
        disc = self.expr()
        self.expect(")")
        self.expect("{")
        cases = []
        while not self.at("}"):
            if self.at_name("case"):
                self.next()
                test = self.expr()
            else:
                if not self.at_name("default"):
                    self.error("expected case")
                self.next()
                test = None
            self.expect(":")
            body = []
            while not (self.at("}") or self.at_name("case") or self.at_name("default")):
                s = self.statement()
                if s is not None:
                    body.append(s)
            cases.append((test, body))
        self.next()
        return ("switch", disc, cases)

    # -- expressions
    def expr(self):
        e = self.assign()
        if self.at(","):
            seq = [e]
            while self.at(","):
                self.next()
                seq.append(self.assign())
            return ("seq", seq)
        return e

    def is_arrow(self):
        t = self.tok
        if t.kind == "name":
            p = self.peek()
            if t.value == "async" and p.kind in ("name", "punc") and not p.nl:
                if p.kind == "name" and self.peek(2).kind == "punc" and self.peek(2).value == "=>":
                    return True
                if p.kind == "punc" and p.value == "(":
                    save = self.i
                    self.next()
                    ok = self._paren_arrow()
                    self.i = save
                    return ok
            return p.kind == "punc" and p.value == "=>" and t.value != "this"
        if t.kind == "punc" and t.value == "(":
            save = self.i
            ok = self._paren_arrow()
            self.i = save
            return ok
        if t.kind == "punc" and t.value == "<":  # generic arrow
            save = self.i
            try:
                self.skip_angle()
                ok = self.at("(") and self._paren_arrow()
            except SyntaxError:
                ok = False
            self.i = save
            return ok
        return False

    def _paren_arrow(self):
        try:
            self.skip_balanced()
        except SyntaxError:
            return False
        if self.at("=>"):
            return True
        if self.at(":"):
            self.next()
            try:
                self.skip_type()
            except SyntaxError:
                return False
            return self.at("=>")
        return False

    def arrow(self):
        if self.at_name("async"):
            self.next()
        if self.at("<"):
            self.skip_angle()
        if self.at_name():
            params = [(("id", self.name()), None, False, None)]
        else:
            params = self.params()
        if self.at(":"):
            self.next()
            self.skip_type()
        self.expect("=>")
        if self.at("{"):
            return ("fn", params, self.block(), True, False, None)
        e = self.assign()
        return ("fn", params, [("ret", e)], True, True, None)

    def assign(self):
        if self.is_arrow():
            return self.arrow()
        left = self.cond()
        t = self.tok
        if t.kind == "punc" and t.value in ASSIGN_OPS:
            self.next()
            right = self.assign()
            return ("asg", t.value, self.to_pattern(left) if t.value == "=" else left, right)
        return left

    def to_pattern(self, e):
        """An assignment target written as an expression -> a pattern where it is one."""
        k = e[0]
        if k == "arr":
            elems, rest = [], None
            for x in e[1]:
                if x is None:
                    elems.append(None)
                elif x[0] == "spread":
                    rest = self.to_pattern(x[1])
                elif x[0] == "asg" and x[1] == "=":
                    elems.append((self.to_pattern(x[2]), x[3]))
                else:
                    elems.append((self.to_pattern(x), None))
            return ("apat", elems, rest)
        if k == "obj":
            props, rest = [], None
            for p in e[1]:
                if p[0] == "spread":
                    rest = self.to_pattern(p[1])
                elif p[0] == "kv":
                    v = p[2]
                    if v[0] == "asg" and v[1] == "=":
                        props.append((p[1], self.to_pattern(v[2]), v[3]))
                    else:
                        props.append((p[1], self.to_pattern(v), None))
                else:
                    self.error("unsupported object pattern")
            return ("opat", props, rest)
        return e

    def cond(self):
        c = self.binary(0)
        if self.at("?"):
            self.next()
            a = self.assign()
            self.expect(":")
            b = self.assign()
            return ("cond", c, a, b)
        return c

    def binary(self, minp):
        left = self.unary()
        while True:
            t = self.tok
            if t.kind == "name" and t.value in ("as", "satisfies") and not t.nl:
                if 8 < minp:
                    break
                self.next()
                self.skip_type()
                continue
            op = t.value if t.kind == "punc" or (t.kind == "name" and t.value in ("instanceof", "in")) else None
            p = BINPREC.get(op)
            if p is None or p < minp:
                break
            self.next()
            right = self.binary(p if op == "**" else p + 1)
            left = ("log", op, left, right) if op in ("&&", "||", "??") else ("bin", op, left, right)
        return left

    def unary(self):
        t = self.tok
        if t.kind == "punc" and t.value in ("!", "-", "+", "~"):
            self.next()
            return ("un", t.value, self.unary())
        if t.kind == "punc" and t.value in ("++", "--"):
            self.next()
            return ("upd", t.value, True, self.unary())
        if t.kind == "name" and t.value in ("typeof", "void", "delete", "await"):
            p = self.peek()
            if not (p.kind == "punc" and p.value in (")", ",", ";", ".", "=")):
                self.next()
                return ("un", t.value, self.unary())
        if t.kind == "punc" and t.value == "<" and self.peek().kind == "name":  # <T>x cast
            save = self.i
            try:
                self.skip_angle()
                return self.unary()
            except SyntaxError:
                self.i = save
        e = self.call_member()
        t = self.tok
        if t.kind == "punc" and t.value in ("++", "--") and not t.nl:
            self.next()
            return ("upd", t.value, False, e)
        return e

    def args(self):
        self.expect("(")
        out = []
        while not self.at(")"):
            if self.at("..."):
                self.next()
                out.append(("spread", self.assign()))
            else:
                out.append(self.assign())
            if self.at(","):
                self.next()
        self.next()
        return out

    def call_member(self, no_call=False):
        if self.at_name("new"):
            self.next()
            if self.at("."):
                self.error("new.target is not supported")
            callee = self.call_member(no_call=True)
            if self.at("<"):
                self.skip_angle()
            args = self.args() if self.at("(") else []
            e = ("new", callee, args)
        else:
            e = self.primary()
        while True:
            t = self.tok
            if t.kind != "punc":
                break
            v = t.value
            if v == ".":
                self.next()
                if self.at("#"):
                    self.next()
                    e = ("mem", e, "_p_" + self.name(), False)
                else:
                    e = ("mem", e, self.next().value, False)
            elif v == "?.":
                self.next()
                if self.at("("):
                    e = ("call", e, self.args(), True)
                elif self.at("["):
                    self.next()
                    x = self.expr()
                    self.expect("]")
                    e = ("idx", e, x, True)
                else:
                    e = ("mem", e, self.next().value, True)
            elif v == "[":
                self.next()
                x = self.expr()
                self.expect("]")
                e = ("idx", e, x, False)
            elif v == "(" and not no_call:
                e = ("call", e, self.args(), False)
            elif v == "!":
                self.next()
            elif v == "<" and not no_call and e[0] in ("id", "mem"):
                save = self.i
                try:
                    self.skip_angle()
                    if self.at("("):
                        continue
                except SyntaxError:
                    pass
                self.i = save
                break
            else:
                break
        return e

    def primary(self):
        t = self.tok
        if t.kind == "num":
            self.next()
            return ("num", t.value)
        if t.kind == "str":
            self.next()
            return ("str", t.value)
        if t.kind == "tmpl":
            self.next()
            strs, srcs = t.value
            return ("tmpl", strs, [Parser(s, self.fname).expr() for s in srcs])
        if t.kind == "punc":
            if t.value == "(":
                self.next()
                e = self.expr()
                self.expect(")")
                return ("paren", e)
            if t.value == "[":
                self.next()
                elems = []
                while not self.at("]"):
                    if self.at(","):
                        self.next()
                        elems.append(("id", "undefined"))
                        continue
                    if self.at("..."):
                        self.next()
                        elems.append(("spread", self.assign()))
                    else:
                        elems.append(self.assign())
                    if self.at(","):
                        self.next()
                self.next()
                return ("arr", elems)
            if t.value == "{":
                return self.object_literal()
            if t.value == "/":
                self.error("regular expression literals are not supported")
        if t.kind == "name":
            v = t.value
            if v == "function":
                self.next()
                name = self.name() if self.at_name() else None
                return self.function_rest(name)
            if v == "class":
                return self.class_decl(expr=True)
            if v == "async" and self.peek().kind == "name" and self.peek().value == "function":
                self.next()
                return self.primary()
            self.next()
            if v == "this":
                return ("this",)
            if v == "super":
                return ("super",)
            return ("id", v)
        self.error("unexpected token")

    def object_literal(self):
        self.expect("{")
        props = []
        while not self.at("}"):
            if self.at("..."):
                self.next()
                props.append(("spread", self.assign()))
            else:
                kind = None
                if (self.at_name("get") or self.at_name("set") or self.at_name("async")) and \
                        self.peek().kind in ("name", "str", "num"):
                    kind = self.next().value
                t = self.next()
                if t.kind == "punc" and t.value == "[":
                    key = self.assign()
                    self.expect("]")
                    computed = True
                else:
                    key = str(t.value) if t.kind != "num" else _js_str(t.value)
                    computed = False
                if self.at("(") or self.at("<"):
                    f = self.function_rest(None if computed else key)
                    if kind in ("get", "set"):
                        props.append((kind, key, f))
                    else:
                        props.append(("ckv" if computed else "kv", key, f))
                elif self.at(":"):
                    self.next()
                    props.append(("ckv" if computed else "kv", key, self.assign()))
                elif self.at("="):  # shorthand with a default (a pattern)
                    self.next()
                    props.append(("kv", key, ("asg", "=", ("id", key), self.assign())))
                else:
                    props.append(("kv", key, ("id", key)))
            if self.at(","):
                self.next()
        self.next()
        return ("obj", props)


# ---------------------------------------------------------------------------
# runtime: JavaScript semantics the generated Python calls into
# ---------------------------------------------------------------------------

_INF = float("inf")
_NAN = float("nan")


def _to_int32(v):
    if type(v) is not int:
        if v is None or v != v or v in (_INF, -_INF):
            return 0
        if isinstance(v, bool):
            v = int(v)
        elif isinstance(v, str):
            return _to_int32(_js_num(v))
        else:
            v = int(v)  # truncates toward zero
    v &= 0xFFFFFFFF
    return v - 0x100000000 if v & 0x80000000 else v


def _to_uint32(v):
    return _to_int32(v) & 0xFFFFFFFF


def _js_num(v):
    if isinstance(v, bool):
        return int(v)
    if isinstance(v, (int, float)):
        return v
    if v is None:
        return _NAN
    if isinstance(v, str):
        s = v.strip()
        if s == "":
            return 0
        try:
            x = float(s) if not s.lower().startswith("0x") else int(s, 16)
            return int(x) if isinstance(x, float) and x.is_integer() and abs(x) < 2 ** 53 else x
        except ValueError:
            return _NAN
    return _NAN


def _js_div(a, b):
    if type(a) is int and type(b) is int and b != 0 and a % b == 0:
        return a // b
    a, b = float(a), float(b)
    if b == 0.0:
        if a != a or a == 0.0:
            return _NAN
        return _INF if (a > 0) == (math.copysign(1.0, b) > 0) else -_INF
    return a / b


def _js_mod(a, b):
    if type(a) is int and type(b) is int and b != 0:
        r = abs(a) % abs(b)
        return -r if a < 0 else r
    a, b = float(a), float(b)
    if b == 0.0 or a != a or b != b or a in (_INF, -_INF):
        return _NAN
    if b in (_INF, -_INF):
        return a
    return math.fmod(a, b)


def _js_pow(a, b):
    try:
        r = a ** b
        return r if not isinstance(r, complex) else _NAN
    except (OverflowError, ZeroDivisionError):
        return _INF


def _js_band(a, b):
    return _to_int32(_to_int32(a) & _to_int32(b))


def _js_bor(a, b):
    return _to_int32(_to_int32(a) | _to_int32(b))


def _js_bxor(a, b):
    return _to_int32(_to_int32(a) ^ _to_int32(b))


def _js_bnot(a):
    return _to_int32(~_to_int32(a))


def _js_shl(a, b):
    return _to_int32(_to_int32(a) << (_to_uint32(b) & 31))


def _js_sar(a, b):
    return _to_int32(a) >> (_to_uint32(b) & 31)


def _js_shr(a, b):
    return _to_uint32(a) >> (_to_uint32(b) & 31)


_PRIM = (int, float, str, bool, type(None))


def _js_seq(a, b):
    if isinstance(a, _PRIM) and isinstance(b, _PRIM):
        if isinstance(a, bool) != isinstance(b, bool) or isinstance(a, str) != isinstance(b, str):
            return False
        return a == b
    return a is b


def _js_typeof(v):
    if v is None:
        return "undefined"
    if isinstance(v, bool):
        return "boolean"
    if isinstance(v, (int, float)):
        return "number"
    if isinstance(v, str):
        return "string"
    if callable(v) and not isinstance(v, _JSObject):
        return "function"
    return "object"


def _js_str(v):
    if v is None:
        return "undefined"
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, float):
        if v != v:
            return "NaN"
        if v in (_INF, -_INF):
            return "Infinity" if v > 0 else "-Infinity"
        if v.is_integer() and abs(v) < 1e21:
            return str(int(v))
        return re.sub(r"e([+-])0*(\d)", r"e\1\2", repr(v))
    if isinstance(v, str):
        return v
    if isinstance(v, (list, array.array)):
        return ",".join("" if x is None else _js_str(x) for x in v)
    if isinstance(v, BaseException):
        return f"{type(v).__name__}: {getattr(v, 'message', '')}"
    return "[object Object]"


def _js_tmpl(strs, vals):
    out = [strs[0]]
    for s, v in zip(strs[1:], vals):
        out.append(_js_str(v))
        out.append(s)
    return "".join(out)


def _js_add(a, b):
    if isinstance(a, str) or isinstance(b, str):
        return _js_str(a) + _js_str(b)
    return a + b


def _raise_loop(b):
    raise ValueError(f"loop bound {b!r} is not finite")


def _js_end(b):
    if type(b) is int:
        return b
    return math.ceil(b) if b == b and b not in (_INF, -_INF) else _raise_loop(b)


def _js_end_le(b):
    return b + 1 if type(b) is int else math.floor(b) + 1


def _js_end_gt(b):
    return b if type(b) is int else math.floor(b)


def _js_end_ge(b):
    return b - 1 if type(b) is int else math.ceil(b) - 1


def _js_start(a):
    if type(a) is int:
        return a
    if isinstance(a, float) and a.is_integer():
        return int(a)
    raise ValueError(f"loop start {a!r} is not an integer")


def _js_length(x):
    if isinstance(x, (list, array.array, str)):
        return len(x)
    return x.length


def _key(k):
    return k if isinstance(k, str) else _js_str(k)


def _js_in(k, obj):
    if isinstance(obj, _JSObject):
        return _key(k) in obj.__dict__
    if isinstance(obj, (list, array.array)):
        return isinstance(k, (int, float)) and 0 <= k < len(obj)
    return hasattr(obj, _key(k))


def _js_spread(x):
    if isinstance(x, _JSObject):
        raise TypeError("spread of a non-iterable object")
    return list(x)


def _js_set_attr(obj, name, v):
    setattr(obj, name, v)
    return v


def _js_set_item(obj, key, v):
    obj[key] = v
    return v


def _js_upd_attr(obj, name, delta, prefix):
    old = getattr(obj, name)
    setattr(obj, name, old + delta)
    return old + delta if prefix else old


def _js_upd_item(obj, key, delta, prefix):
    old = obj[key]
    obj[key] = old + delta
    return old + delta if prefix else old


def _js_delete(obj, key):
    try:
        delattr(obj, _key(key))
    except AttributeError:
        pass
    return True


class _JSError(Exception):
    def __init__(self, message=None, *rest):
        super().__init__(message)
        self.message = "" if message is None else _js_str(message)
        self.name = type(self).__name__

    def __str__(self):
        return f"{self.name}: {self.message}"


class _JSThrow(Exception):
    """A thrown value that is not an Error."""

    def __init__(self, value):
        super().__init__(_js_str(value))
        self.value = value


def _js_throw(v):
    return v if isinstance(v, BaseException) else _JSThrow(v)


def _js_caught(e):
    return e.value if isinstance(e, _JSThrow) else e


class Error(_JSError):
    pass


class RangeError(_JSError):
    pass


class TypeError_(_JSError):
    pass


class _JSObject:
    """A plain JavaScript object: properties are attributes; missing ones are undefined."""

    def __init__(self, props=()):
        d = self.__dict__
        for k, v in props:
            d[k] = v

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return None

    def __getitem__(self, k):
        return self.__dict__.get(_key(k))

    def __setitem__(self, k, v):
        self.__dict__[_key(k)] = v

    def __bool__(self):
        return True

    def __repr__(self):
        return "{" + ", ".join(f"{k}: {v!r}" for k, v in self.__dict__.items()) + "}"


class _Spread:
    __slots__ = ("v",)


def _js_obj(props):
    o = _JSObject()
    d = o.__dict__
    for k, v in props:
        if k is _Spread:
            if isinstance(v, _JSObject):
                d.update(v.__dict__)
            elif isinstance(v, (list, array.array, str)):
                for i, x in enumerate(v):
                    d[str(i)] = x
            elif v is not None and not isinstance(v, _Stub):
                d.update({_key(a): b for a, b in vars(v).items()})
        else:
            d[_key(k)] = v
    return o


def _rel(v, n, default):
    if v is None:
        return default
    v = int(v)
    return max(0, n + v) if v < 0 else min(v, n)


class _JSArr(list):
    """A JavaScript Array."""

    def __bool__(self):
        return True

    @property
    def length(self):
        return len(self)

    @length.setter
    def length(self, n):
        if n < len(self):
            del self[n:]
        else:
            self.extend([None] * (n - len(self)))

    def push(self, *xs):
        self.extend(xs)
        return len(self)

    def pop(self, *a):
        return list.pop(self) if self else None

    def shift(self):
        return list.pop(self, 0) if self else None

    def unshift(self, *xs):
        self[0:0] = xs
        return len(self)

    def slice(self, a=None, b=None):
        return _JSArr(list.__getitem__(self, slice(_rel(a, len(self), 0), _rel(b, len(self), len(self)))))

    def splice(self, start, count=None, *items):
        s = _rel(start, len(self), 0)
        c = len(self) - s if count is None else max(0, min(int(count), len(self) - s))
        out = _JSArr(list.__getitem__(self, slice(s, s + c)))
        self[s:s + c] = items
        return out

    def concat(self, *xs):
        out = _JSArr(self)
        for x in xs:
            if isinstance(x, list):
                out.extend(x)
            else:
                out.append(x)
        return out

    def map(self, fn, *_):
        return _JSArr(fn(x, i, self) for i, x in enumerate(self))

    def filter(self, fn, *_):
        return _JSArr(x for i, x in enumerate(self) if fn(x, i, self))

    def forEach(self, fn, *_):
        for i, x in enumerate(self):
            fn(x, i, self)

    def reduce(self, fn, *init):
        it = iter(enumerate(self))
        if init:
            acc = init[0]
        else:
            _, acc = next(it)
        for i, x in it:
            acc = fn(acc, x, i, self)
        return acc

    def find(self, fn, *_):
        for i, x in enumerate(self):
            if fn(x, i, self):
                return x
        return None

    def findIndex(self, fn, *_):
        for i, x in enumerate(self):
            if fn(x, i, self):
                return i
        return -1

    def some(self, fn, *_):
        return any(fn(x, i, self) for i, x in enumerate(self))

    def every(self, fn, *_):
        return all(fn(x, i, self) for i, x in enumerate(self))

    def includes(self, v, *_):
        return any(_js_seq(x, v) or (x != x and v != v) for x in self)

    def indexOf(self, v, *_):
        for i, x in enumerate(self):
            if _js_seq(x, v):
                return i
        return -1

    def join(self, sep=","):
        return sep.join("" if x is None else _js_str(x) for x in self)

    def fill(self, v, a=None, b=None):
        for i in range(_rel(a, len(self), 0), _rel(b, len(self), len(self))):
            self[i] = v
        return self

    def reverse(self):
        list.reverse(self)
        return self

    def sort(self, cmp=None):
        if cmp is None:
            list.sort(self, key=_js_str)
        else:
            list.sort(self, key=functools.cmp_to_key(lambda x, y: (lambda r: -1 if r < 0 else (1 if r > 0 else 0))(cmp(x, y))))
        return self

    def keys(self):
        return iter(range(len(self)))

    def values(self):
        return iter(self)

    def entries(self):
        return (_JSArr((i, x)) for i, x in enumerate(self))

    def at(self, i):
        i = int(i)
        return self[i] if -len(self) <= i < len(self) else None


class Array(_JSArr):
    def __init__(self, *args):
        if len(args) == 1 and isinstance(args[0], (int, float)) and not isinstance(args[0], bool):
            super().__init__([None] * int(args[0]))
        else:
            super().__init__(args)

    @staticmethod
    def isArray(x):
        return isinstance(x, list)

    @staticmethod
    def of(*xs):
        return _JSArr(xs)


def _array_from(src, fn=None, *_):
    if isinstance(src, _JSObject):
        n = int(src.length or 0)
        items = [src[i] for i in range(n)]
    elif isinstance(src, _JSMap):
        items = [_JSArr(e) for e in src._d.items()]
    elif isinstance(src, _TypedView):
        items = src._mv.tolist()
    else:
        items = list(src)
    if fn is not None:
        items = [fn(x, i) for i, x in enumerate(items)]
    return items


setattr(Array, "from", staticmethod(lambda src, fn=None, *_: _JSArr(_array_from(src, fn))))


class _TypedBase(array.array):
    def __bool__(self):
        return True

    @property
    def length(self):
        return len(self)

    def fill(self, v, a=None, b=None):
        a, b = _rel(a, len(self), 0), _rel(b, len(self), len(self))
        if b > a:
            self[a:b] = type(self)([v] * (b - a))
        return self

    def set(self, src, off=0):
        off = int(off or 0)
        src = list(src)
        if off + len(src) > len(self):
            raise RangeError("offset is out of bounds")
        self[off:off + len(src)] = type(self)(src)

    def subarray(self, a=None, b=None):
        """A copy that refuses writes: in JavaScript a subarray aliases its parent, so a write through
        it would be lost here; reads (the only use in the files this runs) are exact."""
        out = self.slice(a, b)
        out.__class__ = _read_only(type(self))
        return out

    def slice(self, a=None, b=None):
        return type(self)(list(array.array.__getitem__(self, slice(_rel(a, len(self), 0), _rel(b, len(self), len(self))))))

    def map(self, fn, *_):
        return type(self)([fn(x, i, self) for i, x in enumerate(self)])

    def forEach(self, fn, *_):
        for i, x in enumerate(self):
            fn(x, i, self)

    def every(self, fn, *_):
        return all(fn(x, i, self) for i, x in enumerate(self))

    def some(self, fn, *_):
        return any(fn(x, i, self) for i, x in enumerate(self))

    def reduce(self, fn, *init):
        return _JSArr(self).reduce(fn, *init)

    def indexOf(self, v, *_):
        for i, x in enumerate(self):
            if x == v:
                return i
        return -1

    def includes(self, v, *_):
        return self.indexOf(v) >= 0 or (v != v and any(x != x for x in self))

    def join(self, sep=","):
        return sep.join(_js_str(x) for x in self)

    def filter(self, fn, *_):
        return type(self)([x for i, x in enumerate(self) if fn(x, i, self)])


def _make_typed(name, code, conv):
    def __new__(cls, arg=0, *rest):
        if isinstance(arg, ArrayBuffer):
            return _TypedView(cls, arg, int(rest[0]) if rest and rest[0] is not None else 0,
                              int(rest[1]) if len(rest) > 1 and rest[1] is not None else None)
        if isinstance(arg, (int, float)) and not isinstance(arg, bool):
            n = int(arg)
            if n != arg or n < 0:
                raise RangeError("Invalid typed array length")
            return array.array.__new__(cls, code, bytes(n * array.array(code).itemsize))
        items = _array_from(arg)
        if conv is not None:
            items = [conv(x) for x in items]
        return array.array.__new__(cls, code, items)

    def __init__(self, *a):
        pass

    ns = {"__new__": __new__, "__init__": __init__}
    if conv is not None:
        def __setitem__(self, i, v):
            if isinstance(i, slice):
                array.array.__setitem__(self, i, array.array(code, [conv(x) for x in v]))
            else:
                array.array.__setitem__(self, i, conv(v))
        ns["__setitem__"] = __setitem__
    cls = type(name, (_TypedBase,), ns)
    setattr(cls, "from", classmethod(lambda c, src, fn=None, *_: c(_array_from(src, fn))))
    cls.BYTES_PER_ELEMENT = array.array(code).itemsize
    cls._code = code
    cls._conv = staticmethod(conv) if conv is not None else None
    return cls


class ArrayBuffer:
    """Raw bytes that typed-array views alias (a memoryview of a bytearray or of a typed array's storage)."""

    def __init__(self, n=0, *_):
        self._mv = memoryview(bytearray(int(n))) if not isinstance(n, memoryview) else n

    @property
    def byteLength(self):
        return self._mv.nbytes

    def slice(self, a=None, b=None):
        n = self._mv.nbytes
        return ArrayBuffer(memoryview(bytearray(self._mv[_rel(a, n, 0):_rel(b, n, n)])))

    def __bool__(self):
        return True


def _buffer_of(self):
    return ArrayBuffer(memoryview(self).cast("B"))


_TypedBase.buffer = property(_buffer_of)
_TypedBase.byteOffset = property(lambda self: 0)
_TypedBase.byteLength = property(lambda self: len(self) * self.itemsize)


class _TypedView:
    """A typed array over part of an ArrayBuffer: reads and writes reach the buffer, as in JavaScript."""

    def __init__(self, cls, buf, off, n):
        size = cls.BYTES_PER_ELEMENT
        if off % size:
            raise RangeError(f"start offset of {cls.__name__} should be a multiple of {size}")
        if n is None:
            if (buf.byteLength - off) % size:
                raise RangeError(f"byte length of {cls.__name__} should be a multiple of {size}")
            n = (buf.byteLength - off) // size
        if off + n * size > buf.byteLength:
            raise RangeError("invalid typed array length")
        self._cls, self._buf, self._off, self._n = cls, buf, off, n
        self._mv = buf._mv[off:off + n * size].cast(cls._code)
        self._conv = cls._conv

    def __len__(self):
        return self._n

    def __iter__(self):
        return iter(self._mv.tolist())

    def __getitem__(self, i):
        if isinstance(i, slice):
            return self._mv.tolist()[i]
        return self._mv[i]

    def __setitem__(self, i, v):
        conv = self._conv
        if isinstance(i, slice):
            vals = list(v)
            self._mv[i] = memoryview(array.array(self._cls._code, [conv(x) for x in vals] if conv else vals)).cast(
                "B").cast(self._cls._code)
        else:
            self._mv[i] = conv(v) if conv else v

    def __bool__(self):
        return True

    length = property(lambda self: self._n)
    buffer = property(lambda self: self._buf)
    byteOffset = property(lambda self: self._off)
    byteLength = property(lambda self: self._n * self._cls.BYTES_PER_ELEMENT)

    def set(self, src, off=0):
        off = int(off or 0)
        src = list(src)
        if off + len(src) > self._n:
            raise RangeError("offset is out of bounds")
        for k, x in enumerate(src):
            self[off + k] = x

    def subarray(self, a=None, b=None):
        a, b = _rel(a, self._n, 0), _rel(b, self._n, self._n)
        size = self._cls.BYTES_PER_ELEMENT
        return _TypedView(self._cls, self._buf, self._off + a * size, max(0, b - a))

    def slice(self, a=None, b=None):
        return self._cls(self[_rel(a, self._n, 0):_rel(b, self._n, self._n)])

    def fill(self, v, a=None, b=None):
        for k in range(_rel(a, self._n, 0), _rel(b, self._n, self._n)):
            self[k] = v
        return self


@functools.lru_cache(maxsize=None)
def _read_only(cls):
    def refuse(self, *a):
        raise NotImplementedError("a write through a subarray would not reach its parent")
    return type(cls.__name__, (cls,), {"__setitem__": refuse, "fill": refuse, "set": refuse})


def _to_f32(v):
    return struct.unpack("f", struct.pack("f", v))[0]


Float32Array = _make_typed("Float32Array", "f", None)
Float64Array = _make_typed("Float64Array", "d", None)
Uint32Array = _make_typed("Uint32Array", "I", _to_uint32)
Int32Array = _make_typed("Int32Array", "i", _to_int32)
Uint16Array = _make_typed("Uint16Array", "H", lambda v: _to_int32(v) & 0xFFFF)
Int16Array = _make_typed("Int16Array", "h", lambda v: ((_to_int32(v) & 0xFFFF) ^ 0x8000) - 0x8000)
Uint8Array = _make_typed("Uint8Array", "B", lambda v: _to_int32(v) & 0xFF)
Int8Array = _make_typed("Int8Array", "b", lambda v: ((_to_int32(v) & 0xFF) ^ 0x80) - 0x80)


class _JSMap:
    def __init__(self, entries=None, *_):
        self._d = {}
        if entries is not None:
            for k, v in entries:
                self._d[k] = v

    def get(self, k):
        return self._d.get(k)

    def set(self, k, v):
        self._d[k] = v
        return self

    def has(self, k):
        return k in self._d

    def delete(self, k):
        return self._d.pop(k, _Spread) is not _Spread

    @property
    def size(self):
        return len(self._d)

    def keys(self):
        return iter(list(self._d))

    def values(self):
        return iter(list(self._d.values()))

    def entries(self):
        return (_JSArr(kv) for kv in list(self._d.items()))

    def __iter__(self):
        return self.entries()

    def forEach(self, fn, *_):
        for k, v in list(self._d.items()):
            fn(v, k, self)

    def __bool__(self):
        return True


class _JSSet:
    def __init__(self, items=None, *_):
        self._d = dict.fromkeys(items) if items is not None else {}

    def add(self, k):
        self._d[k] = None
        return self

    def has(self, k):
        return k in self._d

    def delete(self, k):
        return self._d.pop(k, _Spread) is not _Spread

    @property
    def size(self):
        return len(self._d)

    def __iter__(self):
        return iter(list(self._d))

    def values(self):
        return iter(list(self._d))

    def forEach(self, fn, *_):
        for k in list(self._d):
            fn(k, k, self)

    def __bool__(self):
        return True


def _js_max(*xs):
    r = -_INF
    for x in xs:
        x = _js_num(x)
        if x != x:
            return _NAN
        if x > r or (x == 0 and r == 0 and math.copysign(1, r) < 0):
            r = x
    return r


def _js_min(*xs):
    r = _INF
    for x in xs:
        x = _js_num(x)
        if x != x:
            return _NAN
        if x < r or (x == 0 and r == 0 and math.copysign(1, x) < 0):
            r = x
    return r


def _js_exp(x):
    try:
        return math.exp(x)
    except OverflowError:
        return _INF


def _js_log(x):
    if x != x or x < 0:
        return _NAN
    if x == 0:
        return -_INF
    return math.log(x) if x != _INF else _INF


def _js_sqrt(x):
    if x != x or x < 0:
        return _NAN
    return math.sqrt(x)


def _int_if(v):
    return int(v) if v == v and v not in (_INF, -_INF) else v


def _finite(x):
    return x == x and x not in (_INF, -_INF)


def _js_round(x):
    if not _finite(x) or type(x) is int:
        return x
    return _int_if(math.floor(x + 0.5)) if not (-0.5 <= x < 0) else -0.0


def _imul(a, b):
    return _to_int32(_to_int32(a) * _to_int32(b))


def _no_random(*_):
    raise NotImplementedError("Math.random")


def _fn1(f):
    """A one-argument Math function that, as in JavaScript, ignores extra arguments (e.g. `xs.map(Math.abs)`)."""
    return lambda x=None, *_: f(x)


def _fn2(f):
    return lambda x=None, y=None, *_: f(x, y)


def _floor(x):
    return _int_if(math.floor(x)) if _finite(x) else x


def _ceil(x):
    return _int_if(math.ceil(x)) if _finite(x) else x


def _trunc(x):
    return _int_if(math.trunc(x)) if _finite(x) else x


def _sign(x):
    return x if x != x or x == 0 else (1 if x > 0 else -1)


def _log2(x):
    return math.log2(x) if x > 0 else _js_log(x)


def _log10(x):
    return math.log10(x) if x > 0 else _js_log(x)


def _log1p(x):
    return math.log1p(x) if x > -1 else (-_INF if x == -1 else _NAN)


Math = _JSObject((
    ("exp", _fn1(_js_exp)), ("log", _fn1(_js_log)), ("sqrt", _fn1(_js_sqrt)), ("max", _js_max), ("min", _js_min),
    ("abs", _fn1(abs)), ("floor", _fn1(_floor)), ("ceil", _fn1(_ceil)), ("round", _fn1(_js_round)),
    ("trunc", _fn1(_trunc)), ("sign", _fn1(_sign)), ("cos", _fn1(math.cos)), ("sin", _fn1(math.sin)),
    ("tan", _fn1(math.tan)), ("tanh", _fn1(math.tanh)), ("atan", _fn1(math.atan)), ("atan2", _fn2(math.atan2)),
    ("pow", _fn2(_js_pow)), ("hypot", lambda *xs: math.hypot(*xs)), ("log2", _fn1(_log2)), ("log10", _fn1(_log10)),
    ("log1p", _fn1(_log1p)), ("expm1", _fn1(math.expm1)), ("imul", _fn2(_imul)), ("fround", _fn1(_to_f32)),
    ("random", _no_random), ("PI", math.pi), ("E", math.e), ("LN2", math.log(2)), ("SQRT2", math.sqrt(2)),
))

Number = _JSObject((
    ("isInteger", lambda v, *_: isinstance(v, (int, float)) and not isinstance(v, bool) and _finite(v)
     and float(v).is_integer()),
    ("isFinite", lambda v, *_: isinstance(v, (int, float)) and not isinstance(v, bool) and _finite(v)),
    ("isNaN", lambda v, *_: isinstance(v, float) and v != v),
    ("isSafeInteger", lambda v, *_: isinstance(v, (int, float)) and _finite(v) and float(v).is_integer()
     and abs(v) <= 2 ** 53 - 1),
    ("MAX_SAFE_INTEGER", 2 ** 53 - 1), ("MIN_SAFE_INTEGER", -(2 ** 53 - 1)), ("EPSILON", 2.0 ** -52),
    ("POSITIVE_INFINITY", _INF), ("NEGATIVE_INFINITY", -_INF), ("MAX_VALUE", sys.float_info.max),
    ("MIN_VALUE", 5e-324), ("NaN", _NAN),
    ("parseFloat", lambda s, *_: _js_num(s)), ("parseInt", lambda s, b=10, *_: int(str(s).strip(), int(b))),
))

Object = _JSObject((
    ("keys", lambda o, *_: _JSArr(o.__dict__.keys() if isinstance(o, _JSObject) else [str(i) for i in range(len(o))])),
    ("values", lambda o, *_: _JSArr(o.__dict__.values() if isinstance(o, _JSObject) else o)),
    ("entries", lambda o, *_: _JSArr(_JSArr(kv) for kv in o.__dict__.items())),
    ("freeze", lambda o, *_: o), ("isFrozen", lambda o, *_: False),
    ("assign", lambda t, *srcs: ([t.__dict__.update(s.__dict__) for s in srcs if s is not None], t)[1]),
    ("fromEntries", lambda es, *_: _js_obj([(k, v) for k, v in es])),
))

JSON = _JSObject((("stringify", lambda v, *_: _js_str(v)),))


class _Stub:
    """A binding from an absent third-party package: any use yields another stub."""

    def __init__(self, name):
        self._name = name

    def __getattr__(self, k):
        return _Stub(f"{self._name}.{k}")

    def __call__(self, *a, **k):
        return _Stub(f"{self._name}()")

    def __iter__(self):
        return iter(())

    def __repr__(self):
        return f"<stub {self._name}>"


def _js_get(o, k):
    if isinstance(o, _JSObject):
        return o.__dict__.get(k)
    if isinstance(o, (list, array.array, str)):
        if k == "length":
            return len(o)
        return o[int(k)]
    return getattr(o, k, None)


def _js_keys(o):
    if isinstance(o, _JSObject):
        return list(o.__dict__.keys())
    if isinstance(o, (list, array.array, str)):
        return [str(i) for i in range(len(o))]
    return []


def _runtime():
    g = {k: v for k, v in globals().items() if k.startswith(("_js_", "_to_", "_JS", "_Spread", "_Stub", "_key"))}
    g.update(Math=Math, Number=Number, Object=Object, JSON=JSON, Array=Array, Error=Error, RangeError=RangeError,
             TypeError=TypeError_, Map=_JSMap, Set=_JSSet, Float32Array=Float32Array, Float64Array=Float64Array,
             Uint32Array=Uint32Array, Int32Array=Int32Array, Uint16Array=Uint16Array, Int16Array=Int16Array,
             Uint8Array=Uint8Array, Int8Array=Int8Array, ArrayBuffer=ArrayBuffer, Infinity=_INF, NaN=_NAN, undefined=None,
             _R_range=range, _R_getattr=getattr, _R_setattr=setattr, _R_isinstance=isinstance, _R_list=list,
             String=lambda v="", *_: _js_str(v), Boolean=lambda v=None, *_: bool(v),
             isNaN=lambda v, *_: _js_num(v) != _js_num(v),
             isFinite=lambda v, *_: Number.isFinite(_js_num(v)),
             Promise=_JSObject((("resolve", lambda v=None, *_: v), ("all", lambda xs, *_: _JSArr(xs)))),
             console=_JSObject((("log", lambda *a: None), ("warn", lambda *a: None), ("error", lambda *a: None))),
             globalThis=_JSObject(), Symbol=_Stub("Symbol"))
    return g


# ---------------------------------------------------------------------------
# code generation: AST -> Python source
# ---------------------------------------------------------------------------

# JavaScript identifiers renamed in the generated Python: its keywords, and the
# builtins the generated code or its readers could otherwise confuse.
PY_RESERVED = set(keyword.kwlist) | {
    "self", "print", "exec", "len", "range", "type", "super", "object", "list", "dict", "str", "int", "float", "bool",
    "id", "iter", "next", "map", "filter", "sum", "min", "max", "abs", "round", "any", "all", "set", "hash", "input",
    "open", "format", "vars", "slice", "zip", "sorted", "reversed", "enumerate", "property", "staticmethod",
    "classmethod", "callable", "repr", "chr", "ord", "globals"}
JS_CONSTS = {"undefined": "None", "null": "None", "true": "True", "false": "False", "NaN": "_js_NaN",
             "Infinity": "_js_Inf"}


def _pyname(n):
    n = n.replace("$", "_S_")
    if n in PY_RESERVED or n.startswith(("_js_", "_R_", "_t_", "_fn_", "_m_")):
        return n + "_"
    return n


def _attr_ok(n):
    return n.isidentifier() and not keyword.iskeyword(n) and not n.startswith("__")


class Scope:
    def __init__(self, parent, is_func, cls=None):
        self.parent = parent
        self.is_func = is_func
        self.names = {}          # js name -> py name (this block)
        self.func = self if is_func else parent.func
        self.cls = cls if cls is not None else (parent.cls if parent is not None else None)
        self.is_module = False
        if is_func:
            self.used_py = set()     # py names declared in this function
            self.nonlocals = set()
            self.globals = set()

    def lookup(self, n):
        s = self
        while s is not None:
            if n in s.names:
                return s.names[n], s
            s = s.parent
        return None, None


class Gen:
    OPFN = {"/": "_js_div", "%": "_js_mod", "**": "_js_pow", "&": "_js_band", "|": "_js_bor", "^": "_js_bxor",
            "<<": "_js_shl", ">>": "_js_sar", ">>>": "_js_shr"}

    def __init__(self, module_path):
        self.lines = []
        self.tmp = 0
        self.module_path = module_path
        self.scope = Scope(None, True)
        self.scope.is_module = True
        self.pre = []               # hoisted definitions for the statement being generated
        self.loop_updates = []      # per enclosing loop: the update lines a `continue` must run first
        self.ctor_fields = None
        self.pending_fields = None
        self.super_base = None

    # -- helpers
    def t(self, prefix="_t_"):
        self.tmp += 1
        return f"{prefix}{self.tmp}"

    def declare(self, n, scope=None):
        scope = scope or self.scope
        if n in scope.names:
            return scope.names[n]
        existing, _ = scope.lookup(n)
        py = _pyname(n)
        f = scope.func
        if existing is not None or py in f.used_py:
            self.tmp += 1
            py = f"{py}__{self.tmp}"
        scope.names[n] = py
        f.used_py.add(py)
        return py

    def resolve(self, n, assign=False):
        if n in JS_CONSTS:
            return JS_CONSTS[n]
        py, sc = self.scope.lookup(n)
        if py is None:
            return _pyname(n) if n != "TypeError" else n
        if assign and sc.func is not self.scope.func:
            if sc.func.is_module:
                self.scope.func.globals.add(py)
            else:
                self.scope.func.nonlocals.add(py)
        return py

    def emit(self, ind, line):
        self.lines.append("    " * ind + line)

    def flush_pre(self, ind):
        for block in self.pre:
            for line in block:
                self.lines.append("    " * ind + line)
        self.pre = []

    def collect_decls(self, stmts):
        """Names declared directly in a block (declared on entry so forward references resolve)."""
        out = []
        for s in stmts:
            k = s[0]
            if k == "var":
                for pat, _ in s[2]:
                    out.extend(self.pat_names(pat))
            elif k in ("fundecl", "classdecl"):
                out.append(s[1])
            elif k == "block_seq":
                out.extend(self.collect_decls(s[1]))
        return out

    def pat_names(self, p):
        k = p[0]
        if k == "id":
            return [p[1]]
        r = []
        if k == "opat":
            for _, sub, _ in p[1]:
                r.extend(self.pat_names(sub))
        elif k == "apat":
            for e in p[1]:
                if e:
                    r.extend(self.pat_names(e[0]))
        if k in ("opat", "apat") and p[2]:
            r.extend(self.pat_names(p[2]))
        return r

    # -- module
    def module(self, body):
        self.emit(0, "_js_NaN = float('nan'); _js_Inf = float('inf')")
        for n in self.collect_decls(body):
            self.declare(n)
        self.block_body(body, 0)
        return "\n".join(self.lines) + "\n"

    def block_body(self, stmts, ind):
        """Function declarations first (hoisting), then the rest in order."""
        funs = [s for s in stmts if s[0] == "fundecl"]
        rest = [s for s in stmts if s[0] != "fundecl"]
        start = len(self.lines)
        for s in funs + rest:
            self.stmt(s, ind)
        if len(self.lines) == start:
            self.emit(ind, "pass")

    def in_block(self, stmts, ind):
        self.scope = Scope(self.scope, False)
        for n in self.collect_decls(stmts):
            self.declare(n)
        self.block_body(stmts, ind)
        self.scope = self.scope.parent

    def sub(self, s, ind):
        """A statement that is the body of if/for/while."""
        self.in_block(s[1] if s is not None and s[0] == "block" else ([s] if s is not None else []), ind)

    # -- statements
    def stmt(self, s, ind):
        getattr(self, "s_" + s[0])(s, ind)

    def s_block(self, s, ind):
        self.in_block(s[1], ind)

    def s_block_seq(self, s, ind):
        for x in s[1]:
            self.stmt(x, ind)

    def s_var(self, s, ind):
        for pat, init in s[2]:
            if pat[0] == "id":
                py = self.declare(pat[1])
                v = self.expr(init) if init is not None else "None"
                self.flush_pre(ind)
                self.emit(ind, f"{py} = {v}")
            else:
                for n in self.pat_names(pat):
                    self.declare(n)
                v = self.expr(init)
                self.flush_pre(ind)
                tmp = self.t()
                self.emit(ind, f"{tmp} = {v}")
                self.assign_pattern(pat, tmp, ind, declare=True)

    def assign_pattern(self, pat, src, ind, declare=False):
        k = pat[0]
        if k == "id":
            py = self.declare(pat[1]) if declare else self.resolve(pat[1], assign=True)
            self.emit(ind, f"{py} = {src}")
        elif k == "opat":
            for key, sub, dflt in pat[1]:
                acc = f"_js_get({src}, {key!r})"
                if dflt is not None:
                    tmp = self.t()
                    self.emit(ind, f"{tmp} = {acc}")
                    d = self.expr(dflt)
                    self.flush_pre(ind)
                    self.emit(ind, f"if {tmp} is None: {tmp} = {d}")
                    acc = tmp
                if sub[0] == "id":
                    self.assign_pattern(sub, acc, ind, declare)
                else:
                    tmp = self.t()
                    self.emit(ind, f"{tmp} = {acc}")
                    self.assign_pattern(sub, tmp, ind, declare)
            if pat[2] is not None:
                keys = tuple(p[0] for p in pat[1])
                tmp = self.t()
                self.emit(ind, f"{tmp} = _js_obj((k, v) for k, v in {src}.__dict__.items() if k not in {keys!r})")
                self.assign_pattern(pat[2], tmp, ind, declare)
        elif k == "apat":
            lst = self.t()
            self.emit(ind, f"{lst} = _R_list({src})")
            for i, e in enumerate(pat[1]):
                if e is None:
                    continue
                sub, dflt = e
                acc = f"({lst}[{i}] if {i} < len({lst}) else None)"
                if dflt is not None:
                    tmp = self.t()
                    self.emit(ind, f"{tmp} = {acc}")
                    d = self.expr(dflt)
                    self.flush_pre(ind)
                    self.emit(ind, f"if {tmp} is None: {tmp} = {d}")
                    acc = tmp
                tmp = self.t()
                self.emit(ind, f"{tmp} = {acc}")
                self.assign_pattern(sub, tmp, ind, declare)
            if pat[2] is not None:
                tmp = self.t()
                self.emit(ind, f"{tmp} = _JSArr({lst}[{len(pat[1])}:])")
                self.assign_pattern(pat[2], tmp, ind, declare)
        else:  # an expression target (member / index)
            self.emit(ind, f"{self.target(pat)} = {src}")

    def s_fundecl(self, s, ind):
        self.function(s[2], self.resolve(s[1]), ind)

    def s_classdecl(self, s, ind):
        self.klass(s[2], self.resolve(s[1]), ind)

    def s_expr(self, s, ind):
        e = s[1]
        while e[0] == "paren":
            e = e[1]
        if e[0] == "asg":
            self.assign_stmt(e, ind)
            return
        if e[0] == "upd":
            tgt = e[3]
            d = "1" if e[1] == "++" else "-1"
            t = self.resolve(tgt[1], assign=True) if tgt[0] == "id" else self.target(tgt)
            self.flush_pre(ind)
            self.emit(ind, f"{t} += {d}")
            return
        if e[0] == "seq":
            for x in e[1]:
                self.s_expr(("expr", x), ind)
            return
        v = self.expr(e)
        self.flush_pre(ind)
        self.emit(ind, v)
        if e[0] == "call" and e[1] == ("super",):
            for line in self.pending_fields or []:  # fields initialise right after super() returns
                self.emit(ind, line)
            self.pending_fields = None

    def assign_stmt(self, e, ind):
        _, op, tgt, val = e
        if op == "=" and tgt[0] in ("apat", "opat"):
            v = self.expr(val)
            self.flush_pre(ind)
            tmp = self.t()
            self.emit(ind, f"{tmp} = {v}")
            self.assign_pattern(tgt, tmp, ind)
            return
        if op == "=" and val[0] == "asg":  # a = b = c
            self.assign_stmt(val, ind)
            inner = val
            while inner[0] == "asg":
                last_target = inner[2]
                inner = inner[3]
            src = self.expr(last_target)
            t = self.target(tgt)
            self.flush_pre(ind)
            self.emit(ind, f"{t} = {src}")
            return
        v = self.expr(val)
        t = self.target(tgt)
        self.flush_pre(ind)
        if op == "=":
            self.emit(ind, f"{t} = {v}")
        elif op in ("+=", "-=", "*="):
            if op == "+=" and not self.numeric(val):
                self.emit(ind, f"{t} = _js_add({t}, {v})")
            else:
                self.emit(ind, f"{t} {op} {v}")
        elif op == "??=":
            self.emit(ind, f"if {t} is None: {t} = {v}")
        elif op == "||=":
            self.emit(ind, f"if not {t}: {t} = {v}")
        elif op == "&&=":
            self.emit(ind, f"if {t}: {t} = {v}")
        else:
            self.emit(ind, f"{t} = {self.OPFN[op[:-1]]}({t}, {v})")

    def numeric(self, e):
        """True when an expression certainly yields a number (so + needs no string check)."""
        k = e[0]
        if k in ("num", "idx", "id"):
            # typed-array reads and identifiers in arithmetic are numbers in this code (strings are built
            # with templates); a string element would raise on the next numeric use, not mis-add silently
            return True
        if k == "bin":
            return e[1] != "+" or (self.numeric(e[2]) and self.numeric(e[3]))
        if k == "un":
            return e[1] in ("-", "+", "~")
        if k == "paren":
            return self.numeric(e[1])
        if k == "call" and e[1][0] == "mem" and e[1][1] == ("id", "Math"):
            return True
        return False

    def target(self, t):
        k = t[0]
        if k == "paren":
            return self.target(t[1])
        if k == "id":
            return self.resolve(t[1], assign=True)
        if k == "mem":
            o = self.expr(t[1])
            n = t[2]
            if _attr_ok(n):
                return f"{o}.{n}"
            return f"{o}.__dict__[{n!r}]"
        if k == "idx":
            return f"{self.expr(t[1])}[{self.expr(t[2])}]"
        raise SyntaxError(f"cannot assign to {t[0]}")

    def s_ret(self, s, ind):
        v = self.expr(s[1]) if s[1] is not None else "None"
        self.flush_pre(ind)
        self.emit(ind, f"return {v}")

    def s_if(self, s, ind):
        c = self.expr(s[1])
        self.flush_pre(ind)
        self.emit(ind, f"if {c}:")
        self.sub(s[2], ind + 1)
        if s[3] is not None:
            self.emit(ind, "else:")
            self.sub(s[3], ind + 1)

    def s_throw(self, s, ind):
        v = self.expr(s[1])
        self.flush_pre(ind)
        self.emit(ind, f"raise _js_throw({v})")

    def s_break(self, s, ind):
        self.emit(ind, "break")

    def s_continue(self, s, ind):
        if self.loop_updates and self.loop_updates[-1] is not None:
            for line in self.loop_updates[-1]:
                self.emit(ind, line)
        self.emit(ind, "continue")

    def assigned_names(self, node, out):
        if isinstance(node, tuple):
            if node and node[0] in ("asg", "upd"):
                tgt = node[2] if node[0] == "asg" else node[3]
                if isinstance(tgt, tuple) and tgt[0] == "id":
                    out.add(tgt[1])
                if isinstance(tgt, tuple) and tgt[0] in ("apat", "opat"):
                    out.update(self.pat_names(tgt))
            if node and node[0] == "call" and node[1][0] == "mem" and node[1][1][0] == "id" and \
                    node[1][2] in ("push", "pop", "splice", "shift", "unshift"):
                out.add(node[1][1][1])
            for x in node:
                self.assigned_names(x, out)
        elif isinstance(node, list):
            for x in node:
                self.assigned_names(x, out)

    def expr_names(self, e, out):
        """Identifiers an expression reads; False when it calls, assigns or defines anything."""
        if isinstance(e, tuple):
            k = e[0] if e else None
            if k == "id":
                out.add(e[1])
                return True
            if k in ("call", "new", "asg", "upd", "fn"):
                return False
            ok = True
            for x in e[1:]:
                if isinstance(x, (tuple, list)):
                    ok = self.expr_names(x, out) and ok
            return ok
        if isinstance(e, list):
            return all(self.expr_names(x, out) for x in e)
        return True

    def range_loop(self, init, test, update, body):
        """`for (let i = a; i < b; i++)` whose body changes neither i nor what b reads -> a Python range."""
        if init is None or init[0] != "var" or init[1] == "var" or len(init[2]) != 1:
            return None
        pat, start = init[2][0]
        if pat[0] != "id" or start is None or test is None or update is None:
            return None
        var = pat[1]
        if test[0] != "bin" or test[1] not in ("<", "<=", ">", ">=") or test[2] != ("id", var):
            return None
        step = None
        if update[0] == "upd" and update[3] == ("id", var):
            step = 1 if update[1] == "++" else -1
        elif update[0] == "asg" and update[1] in ("+=", "-=") and update[2] == ("id", var) and update[3][0] == "num" \
                and type(update[3][1]) is int:
            step = update[3][1] if update[1] == "+=" else -update[3][1]
        if not step or (step > 0) != (test[1] in ("<", "<=")):
            return None
        assigned = set()
        self.assigned_names(body, assigned)
        if var in assigned:
            return None
        reads = set()
        if not self.expr_names(test[3], reads) or reads & assigned:
            return None
        return var, start, test[1], test[3], step

    def s_for(self, s, ind):
        _, init, test, update, body = s
        fast = self.range_loop(init, test, update, body)
        self.scope = Scope(self.scope, False)
        if fast is not None:
            var, start, op, bound, step = fast
            a = self.expr(start)
            py = self.declare(var)
            b = self.expr(bound)
            self.flush_pre(ind)
            end = {"<": f"_js_end({b})", "<=": f"_js_end_le({b})", ">": f"_js_end_gt({b})",
                   ">=": f"_js_end_ge({b})"}[op]
            self.emit(ind, f"for {py} in _R_range(_js_start({a}), {end}{', ' + str(step) if step != 1 else ''}):")
            self.loop_updates.append(None)
            self.sub(body, ind + 1)
            self.loop_updates.pop()
            self.scope = self.scope.parent
            return
        if init is not None:
            self.stmt(init, ind)
        upd_lines = None
        if update is not None:
            save = len(self.lines)
            self.s_expr(("expr", update), 0)
            upd_lines = self.lines[save:]
            del self.lines[save:]
        self.emit(ind, "while True:")
        if test is not None:
            c = self.expr(test)
            self.flush_pre(ind + 1)
            self.emit(ind + 1, f"if not ({c}): break")
        self.loop_updates.append(upd_lines)
        self.sub(body, ind + 1)
        self.loop_updates.pop()
        for line in upd_lines or []:
            self.emit(ind + 1, line)
        self.scope = self.scope.parent

    def s_forof(self, s, ind):
        _, kind, pat, it, body = s
        src = self.expr(it)
        self.flush_pre(ind)
        self.scope = Scope(self.scope, False)
        if pat[0] == "id":
            py = self.declare(pat[1]) if kind is not None else self.resolve(pat[1], assign=True)
            self.emit(ind, f"for {py} in {src}:")
        else:
            tmp = self.t()
            self.emit(ind, f"for {tmp} in {src}:")
            if kind is not None:
                for n in self.pat_names(pat):
                    self.declare(n)
            self.assign_pattern(pat, tmp, ind + 1, declare=kind is not None)
        self.loop_updates.append(None)
        self.sub(body, ind + 1)
        self.loop_updates.pop()
        self.scope = self.scope.parent

    def s_forin(self, s, ind):
        _, kind, pat, it, body = s
        src = self.expr(it)
        self.flush_pre(ind)
        self.scope = Scope(self.scope, False)
        py = self.declare(pat[1]) if kind is not None else self.resolve(pat[1], assign=True)
        self.emit(ind, f"for {py} in _js_keys({src}):")
        self.loop_updates.append(None)
        self.sub(body, ind + 1)
        self.loop_updates.pop()
        self.scope = self.scope.parent

    def s_while(self, s, ind):
        c = self.expr(s[1])
        if self.pre:
            self.emit(ind, "while True:")
            self.flush_pre(ind + 1)
            self.emit(ind + 1, f"if not ({c}): break")
        else:
            self.emit(ind, f"while {c}:")
        self.loop_updates.append(None)
        self.sub(s[2], ind + 1)
        self.loop_updates.pop()

    def s_dowhile(self, s, ind):
        self.emit(ind, "while True:")
        self.loop_updates.append(None)
        self.sub(s[1], ind + 1)
        self.loop_updates.pop()
        c = self.expr(s[2])
        self.flush_pre(ind + 1)
        self.emit(ind + 1, f"if not ({c}): break")

    def s_try(self, s, ind):
        _, blk, param, handler, fin = s
        self.emit(ind, "try:")
        self.in_block(blk, ind + 1)
        if handler is not None:
            ev = self.t()
            self.emit(ind, f"except Exception as {ev}:")
            self.scope = Scope(self.scope, False)
            if param is not None:
                if param[0] == "id":
                    py = self.declare(param[1])
                    self.emit(ind + 1, f"{py} = _js_caught({ev})")
                else:
                    for n in self.pat_names(param):
                        self.declare(n)
                    self.assign_pattern(param, f"_js_caught({ev})", ind + 1, declare=True)
            self.in_block(handler, ind + 1)
            self.scope = self.scope.parent
        if fin is not None:
            self.emit(ind, "finally:")
            self.in_block(fin, ind + 1)

    def s_switch(self, s, ind):
        _, disc, cases = s
        d = self.expr(disc)
        self.flush_pre(ind)
        sw, hit = self.t(), self.t()
        self.emit(ind, f"{sw} = {d}; {hit} = False")
        self.emit(ind, "while True:")
        default_i = next((i for i, (t, _) in enumerate(cases) if t is None), None)
        for test, body in cases:
            if test is None:
                continue
            c = self.expr(test)
            self.flush_pre(ind + 1)
            self.emit(ind + 1, f"if {hit} or _js_seq({sw}, {c}):")
            self.emit(ind + 2, f"{hit} = True")
            self.loop_updates.append(None)
            self.in_block(body, ind + 2)
            self.loop_updates.pop()
        if default_i is not None:
            for i in range(default_i, len(cases)):
                self.loop_updates.append(None)
                self.in_block(cases[i][1], ind + 1)
                self.loop_updates.pop()
        self.emit(ind + 1, "break")

    def s_import(self, s, ind):
        _, spec, names, default, star = s
        m = self.t("_m_")
        self.emit(ind, f"{m} = _js_import({str(self.module_path)!r}, {spec!r})")
        for n, alias in names:
            py = self.scope.names.get(alias) or self.declare(alias)
            self.emit(ind, f"{py} = {m}[{n!r}]")
        if default is not None:
            py = self.scope.names.get(default) or self.declare(default)
            self.emit(ind, f"{py} = {m}['__default__']")
        if star is not None:
            py = self.scope.names.get(star) or self.declare(star)
            self.emit(ind, f"{py} = _js_namespace({m})")

    def s_exportstar(self, s, ind):
        m = self.t("_m_")
        self.emit(ind, f"{m} = _js_import({str(self.module_path)!r}, {s[1]!r})")
        self.emit(ind, f"_js_export_star(globals(), {m})")

    def s_exportnames(self, s, ind):
        for n, alias in s[1]:
            if alias != n:
                self.emit(ind, f"globals()[{alias!r}] = {self.resolve(n)}")

    # -- functions and classes
    def function(self, fn, pyname, ind, method=False, static=False):
        _, params, body, is_arrow, is_expr, _name = fn
        outer_pre = self.pre
        self.pre = []
        parent = self.scope
        self.scope = Scope(parent, True)
        start = len(self.lines)
        plist, setup = [], []
        if method and not static:
            plist.append("self")
        for pat, dflt, rest, field in params:
            if pat[0] == "id":
                py = self.declare(pat[1])
                if rest:
                    plist.append(f"*{py}")
                    setup.append(("rest", py))
                else:
                    plist.append(f"{py}=None")
                    if dflt is not None:
                        setup.append(("dflt", py, dflt))
                    if field:
                        setup.append(("field", py, field))
            else:
                tmp = self.t()
                plist.append(f"{tmp}=None")
                for n in self.pat_names(pat):
                    self.declare(n)
                setup.append(("pat", tmp, pat, dflt))
        if not any(p.startswith("*") for p in plist):
            plist.append("*_extra")  # JavaScript ignores extra arguments
        for n in self.collect_decls(body):
            self.declare(n)
        for item in setup:
            if item[0] == "rest":
                self.emit(ind + 1, f"{item[1]} = _JSArr({item[1]})")
            elif item[0] == "dflt":
                d = self.expr(item[2])
                self.flush_pre(ind + 1)
                self.emit(ind + 1, f"if {item[1]} is None: {item[1]} = {d}")
            elif item[0] == "field":
                self.emit(ind + 1, f"self.{item[2]} = {item[1]}")
            else:
                _, tmp, pat, dflt = item
                if dflt is not None:
                    d = self.expr(dflt)
                    self.flush_pre(ind + 1)
                    self.emit(ind + 1, f"if {tmp} is None: {tmp} = {d}")
                self.assign_pattern(pat, tmp, ind + 1, declare=True)
        if self.ctor_fields is not None:
            fields, has_super = self.ctor_fields
            self.ctor_fields = None
            if has_super:
                self.pending_fields = fields
            else:
                for line in fields:
                    self.emit(ind + 1, line)
        self.block_body(body, ind + 1)
        body_lines = self.lines[start:]
        del self.lines[start:]
        f = self.scope
        self.scope = parent
        self.pre = outer_pre
        header = []
        if static:
            header.append("    " * ind + "@staticmethod")
        header.append("    " * ind + f"def {pyname}({', '.join(plist)}):")
        decl = []
        if f.nonlocals:
            decl.append("    " * (ind + 1) + "nonlocal " + ", ".join(sorted(f.nonlocals)))
        if f.globals:
            decl.append("    " * (ind + 1) + "global " + ", ".join(sorted(f.globals)))
        self.lines.extend(header + decl + body_lines)
        # names assigned here that live further out than the parent are free in the parent too
        pf = parent.func
        for py in f.nonlocals:
            if py not in pf.used_py and not pf.is_module:
                pf.nonlocals.add(py)
        if not pf.is_module:
            pf.globals.update(f.globals)

    def klass(self, node, pyname, ind):
        _, name, sup, members = node
        base = self.expr(sup) if sup is not None else "_JSObject"
        self.flush_pre(ind)
        self.emit(ind, f"class {pyname}({base}):")
        saved = self.scope
        self.scope = Scope(self.scope, False, cls=pyname)
        fields, statics = [], []
        for kind, mname, init, static in members:
            if kind != "field":
                continue
            if static:
                statics.append((mname, init))
            elif init is not None:
                v = self.expr(init)
                if self.pre:
                    raise SyntaxError("field initialisers with functions are not supported")
                fields.append(f"self.{mname} = {v}" if _attr_ok(mname) else f"self.__dict__[{mname!r}] = {v}")
        wrote = False
        if not any(m[0] == "ctor" for m in members):
            self.emit(ind + 1, "def __init__(self, *args):")
            if sup is not None:
                self.emit(ind + 2, f"{base}.__init__(self, *args)")
            for line in fields:
                self.emit(ind + 2, line)
            self.emit(ind + 2, "pass")
            wrote = True
        for kind, mname, f, static in members:
            if kind == "field":
                continue
            if kind == "ctor":
                self.ctor_fields = (fields, self.calls_super(f[2]))
                self.super_base = base
                self.function(f, "__init__", ind + 1, method=True)
            elif kind == "get":
                py = _pyname(mname)
                self.function(f, py, ind + 1, method=True)
                self.emit(ind + 1, f"{py} = property({py})")
            elif kind == "set":
                py = _pyname(mname)
                self.function(f, f"_set_{py}", ind + 1, method=True)
                self.emit(ind + 1, f"{py} = {py}.setter(_set_{py})")
            else:
                self.function(f, _pyname(mname), ind + 1, method=True, static=static)
            wrote = True
        for mname, init in statics:
            v = self.expr(init) if init is not None else "None"
            self.flush_pre(ind + 1)
            self.emit(ind + 1, f"{_pyname(mname)} = {v}")
            wrote = True
        if not wrote:
            self.emit(ind + 1, "pass")
        self.scope = saved

    def calls_super(self, body):
        found = []

        def walk(n):
            if isinstance(n, tuple):
                if n and n[0] == "call" and n[1] == ("super",):
                    found.append(1)
                for x in n:
                    walk(x)
            elif isinstance(n, list):
                for x in n:
                    walk(x)
        walk(body)
        return bool(found)

    # -- expressions
    def expr(self, e):
        if e[0] in ("mem", "idx", "call"):
            low = self.lower_optional(e)
            if low is not None:
                return low
        return getattr(self, "e_" + e[0])(e)

    def lower_optional(self, e):
        """`a?.b.c(x)`: the first `?.` below this node short-circuits the whole rest of the chain."""
        path, node = [], e
        while node[0] in ("mem", "idx", "call"):
            if node[-1]:  # an optional link: node = (kind, obj, ..., True)
                break
            path.append(node)
            node = node[1]
        else:
            return None
        if not path:
            return None  # this node is the optional link itself (handled by e_mem / e_idx / e_call)
        t = self.t()
        head = (node[0], ("pyraw", t)) + node[2:-1] + (False,)
        for outer in reversed(path):
            head = (outer[0], head) + outer[2:]
        return f"(None if ({t} := {self.expr(node[1])}) is None else {self.expr(head)})"

    def e_pyraw(self, e):
        return e[1]

    def e_paren(self, e):
        return self.expr(e[1])

    def e_num(self, e):
        v = e[1]
        if isinstance(v, float):
            return "_js_Inf" if v == _INF else repr(v)
        return str(v)

    def e_str(self, e):
        return repr(e[1])

    def e_tmpl(self, e):
        vals = ", ".join(self.expr(x) for x in e[2])
        return f"_js_tmpl({tuple(e[1])!r}, ({vals}{',' if len(e[2]) == 1 else ''}))"

    def e_id(self, e):
        return self.resolve(e[1])

    def e_this(self, e):
        return "self"

    def e_super(self, e):
        return "super()"

    def e_arr(self, e):
        parts = [f"*_js_spread({self.expr(x[1])})" if x[0] == "spread" else self.expr(x) for x in e[1]]
        return f"_JSArr([{', '.join(parts)}])"

    def e_obj(self, e):
        parts = []
        for p in e[1]:
            if p[0] == "spread":
                parts.append(f"(_Spread, {self.expr(p[1])})")
            elif p[0] == "kv":
                parts.append(f"({p[1]!r}, {self.expr(p[2])})")
            elif p[0] == "ckv":
                parts.append(f"({self.expr(p[1])}, {self.expr(p[2])})")
            else:
                raise SyntaxError("getters/setters in object literals are not supported")
        return f"_js_obj(({', '.join(parts)}{',' if len(parts) == 1 else ''}))"

    def e_fn(self, e):
        """A function expression or arrow: defined just before the statement that uses it."""
        name = self.t("_fn_")
        save = self.lines
        self.lines = []
        self.function(e, name, 0)
        block = self.lines
        self.lines = save
        self.pre.append(block)
        return name

    def e_class(self, e):
        name = self.t("_fn_")
        save = self.lines
        self.lines = []
        self.klass(e, name, 0)
        block = self.lines
        self.lines = save
        self.pre.append(block)
        return name

    def e_un(self, e):
        op, x = e[1], self.expr(e[2])
        if op == "!":
            return f"(not {x})"
        if op == "-":
            return f"(-{x})"
        if op == "+":
            return f"_js_num({x})"
        if op == "~":
            return f"_js_bnot({x})"
        if op == "typeof":
            if e[2][0] == "id" and self.scope.lookup(e[2][1])[0] is None and e[2][1] not in JS_CONSTS:
                return f"_js_typeof(globals().get({_pyname(e[2][1])!r}))"
            return f"_js_typeof({x})"
        if op == "void":
            return f"({x}, None)[1]"
        if op == "await":
            return x
        if op == "delete":
            t = e[2]
            if t[0] == "mem":
                return f"_js_delete({self.expr(t[1])}, {t[2]!r})"
            return f"_js_delete({self.expr(t[1])}, {self.expr(t[2])})"
        raise SyntaxError(op)

    def e_upd(self, e):
        _, op, prefix, tgt = e
        d = 1 if op == "++" else -1
        if tgt[0] == "id":
            py = self.resolve(tgt[1], assign=True)
            return f"({py} := {py} + {d})" if prefix else f"(({py} := {py} + {d}) - {d})"
        if tgt[0] == "mem":
            return f"_js_upd_attr({self.expr(tgt[1])}, {tgt[2]!r}, {d}, {prefix})"
        return f"_js_upd_item({self.expr(tgt[1])}, {self.expr(tgt[2])}, {d}, {prefix})"

    def e_bin(self, e):
        _, op, l, r = e
        a, b = self.expr(l), self.expr(r)
        if op in ("-", "*"):
            return f"({a} {op} {b})"
        if op == "+":
            if self.numeric(l) and self.numeric(r):
                return f"({a} + {b})"
            return f"_js_add({a}, {b})"
        if op in self.OPFN:
            return f"{self.OPFN[op]}({a}, {b})"
        if op in ("<", ">", "<=", ">="):
            return f"({a} {op} {b})"
        if op in ("===", "==", "!==", "!="):
            neg = op.startswith("!")
            nul = ("undefined", "null")
            if r[0] == "id" and r[1] in nul or l[0] == "id" and l[1] in nul:
                x = a if r[0] == "id" and r[1] in nul else b
                return f"({x} is {'not ' if neg else ''}None)"
            if l[0] in ("num", "str") or r[0] in ("num", "str"):
                return f"({a} {'!=' if neg else '=='} {b})"
            return f"({'not ' if neg else ''}_js_seq({a}, {b}))"
        if op == "instanceof":
            return f"_R_isinstance({a}, {b})"
        if op == "in":
            return f"_js_in({a}, {b})"
        raise SyntaxError(op)

    def e_log(self, e):
        _, op, l, r = e
        a, b = self.expr(l), self.expr(r)
        if op == "&&":
            return f"({a} and {b})"
        if op == "||":
            return f"({a} or {b})"
        t = self.t()
        return f"({t} if ({t} := {a}) is not None else {b})"

    def e_cond(self, e):
        return f"({self.expr(e[2])} if {self.expr(e[1])} else {self.expr(e[3])})"

    def e_asg(self, e):
        _, op, tgt, val = e
        v = self.expr(val)
        if tgt[0] == "id":
            py = self.resolve(tgt[1], assign=True)
            if op == "=":
                return f"({py} := {v})"
            if op in ("+=", "-=", "*="):
                return f"({py} := {py} {op[0]} {v})"
            if op == "??=":
                return f"({py} if {py} is not None else ({py} := {v}))"
            return f"({py} := {self.OPFN[op[:-1]]}({py}, {v}))"
        if op != "=":
            raise SyntaxError("compound assignment to a property inside an expression is not supported")
        if tgt[0] == "mem":
            return f"_js_set_attr({self.expr(tgt[1])}, {tgt[2]!r}, {v})"
        if tgt[0] == "idx":
            return f"_js_set_item({self.expr(tgt[1])}, {self.expr(tgt[2])}, {v})"
        raise SyntaxError("destructuring assignment inside an expression is not supported")

    def e_seq(self, e):
        return "(" + ", ".join(self.expr(x) for x in e[1]) + ")[-1]"

    def e_spread(self, e):
        return f"*_js_spread({self.expr(e[1])})"

    def args(self, args):
        return ", ".join(self.expr(a) for a in args)

    def e_call(self, e):
        _, callee, args, opt = e
        if callee == ("super",):
            return f"{self.super_base}.__init__(self, {self.args(args)})"
        if callee == ("id", "import"):  # a dynamic import: the module's namespace (synchronously)
            return f"_js_namespace(_js_import({str(self.module_path)!r}, {self.args(args)}))"
        if callee[0] == "mem" and callee[1] == ("super",):
            return f"super().{callee[2]}({self.args(args)})"
        if opt:
            t = self.t()
            return f"(None if ({t} := {self.expr(callee)}) is None else {t}({self.args(args)}))"
        return f"{self.expr(callee)}({self.args(args)})"

    def e_new(self, e):
        _, callee, args = e
        return f"{self.expr(callee)}({self.args(args)})"

    def e_mem(self, e):
        _, obj, name, opt = e
        o = self.expr(obj)
        if name == "length":
            acc = "_js_length({})"
        elif _attr_ok(name):
            acc = f"{{}}.{name}"
        else:
            acc = f"_R_getattr({{}}, {name!r})"
        if opt:
            t = self.t()
            return f"(None if ({t} := {o}) is None else {acc.format(t)})"
        return acc.format(o)

    def e_idx(self, e):
        _, obj, x, opt = e
        o, i = self.expr(obj), self.expr(x)
        if opt:
            t = self.t()
            return f"(None if ({t} := {o}) is None else {t}[{i}])"
        return f"{o}[{i}]"


# ---------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------

class _StubModule(dict):
    def __init__(self, spec):
        super().__init__()
        self.spec = spec

    def __missing__(self, k):
        return _Stub(f"{self.spec}:{k}")


class Runner:
    """Loads TypeScript modules from a source tree and runs them. Imports of
    packages outside the tree (third-party, not vendored) bind stubs, except
    those given in `packages` (specifier -> dict of exports)."""

    def __init__(self, packages=None):
        self.modules = {}
        self.sources = {}
        self.packages = dict(packages or {})

    @staticmethod
    def resolve(from_file, spec):
        if not spec.startswith("."):
            return None
        base = Path(from_file).parent / spec
        for cand in (base, base.with_name(base.name + ".ts"), base / "index.ts"):
            if cand.is_file():
                return cand.resolve()
        raise FileNotFoundError(f"cannot resolve {spec!r} from {from_file}")

    def import_(self, from_file, spec):
        if spec in self.packages:
            return self.packages[spec]
        path = self.resolve(from_file, spec)
        return _StubModule(spec) if path is None else self.load(path)

    def translate(self, path):
        src = Path(path).read_text()
        return Gen(path).module(Parser(src, str(path)).program())

    def load(self, path):
        path = Path(path).resolve()
        if path in self.modules:
            return self.modules[path]
        ns = _runtime()
        ns["_js_import"] = self.import_
        ns["_js_namespace"] = lambda m: _js_obj([(k, v) for k, v in m.items() if not k.startswith("_")])
        ns["_js_export_star"] = lambda g, m: g.update({k: v for k, v in m.items()
                                                        if not k.startswith("_") and k not in g})
        ns["__name__"] = f"ts:{path.name}"
        self.modules[path] = ns
        code = self.translate(path)
        self.sources[path] = code
        exec(compile(code, f"<ts {path}>", "exec"), ns)
        return ns


# ---------------------------------------------------------------------------
# bun:test, enough of it to run the reference's CPU unit tests
# ---------------------------------------------------------------------------

class _Expectation(Exception):
    pass


def _deep_equal(a, b):
    if isinstance(a, (list, array.array)) and isinstance(b, (list, array.array)):
        return len(a) == len(b) and all(_deep_equal(x, y) for x, y in zip(a, b))
    if isinstance(a, _JSObject) and isinstance(b, _JSObject):
        ka = {k for k, v in a.__dict__.items() if v is not None}
        kb = {k for k, v in b.__dict__.items() if v is not None}
        return ka == kb and all(_deep_equal(a.__dict__[k], b.__dict__[k]) for k in ka)
    if isinstance(a, float) and isinstance(b, float) and a != a and b != b:
        return True
    return _js_seq(a, b) or (isinstance(a, (int, float)) and isinstance(b, (int, float))
                             and not isinstance(a, bool) and not isinstance(b, bool) and a == b)


class _Expect:
    def __init__(self, value, negate=False):
        self.v = value
        self.negate = negate

    def _check(self, ok, what):
        if bool(ok) == self.negate:
            raise _Expectation(f"expected {_js_str(self.v) if not isinstance(self.v, _JSObject) else self.v!r} "
                               f"{'not ' if self.negate else ''}{what}")

    def toBe(self, x, *_):
        self._check(_js_seq(self.v, x) or (self.v != self.v and x != x), f"to be {x!r}")

    def toEqual(self, x, *_):
        self._check(_deep_equal(self.v, x), f"to equal {x!r}")

    toStrictEqual = toEqual

    def toBeCloseTo(self, x, digits=2, *_):
        self._check(abs(self.v - x) < 10 ** (-digits) / 2, f"to be close to {x!r} ({digits} digits)")

    def toBeGreaterThan(self, x, *_):
        self._check(self.v > x, f"to be > {x!r}")

    def toBeGreaterThanOrEqual(self, x, *_):
        self._check(self.v >= x, f"to be >= {x!r}")

    def toBeLessThan(self, x, *_):
        self._check(self.v < x, f"to be < {x!r}")

    def toBeLessThanOrEqual(self, x, *_):
        self._check(self.v <= x, f"to be <= {x!r}")

    def toHaveLength(self, n, *_):
        self._check(_js_length(self.v) == n, f"to have length {n}")

    def toContain(self, x, *_):
        self._check(any(_js_seq(y, x) for y in self.v) if not isinstance(self.v, str) else x in self.v,
                    f"to contain {x!r}")

    def toBeNull(self, *_):
        self._check(self.v is None, "to be null")

    toBeUndefined = toBeNull

    def toBeDefined(self, *_):
        self._check(self.v is not None, "to be defined")

    def toBeTruthy(self, *_):
        self._check(bool(self.v) and self.v == self.v, "to be truthy")

    def toBeFalsy(self, *_):
        self._check(not (bool(self.v) and self.v == self.v), "to be falsy")

    def toBeNaN(self, *_):
        self._check(isinstance(self.v, float) and self.v != self.v, "to be NaN")

    def toThrow(self, what=None, *_):
        try:
            self.v()
            thrown = None
        except _Expectation:
            raise
        except Exception as e:  # noqa: BLE001 - any thrown value counts
            thrown = e
        ok = thrown is not None
        if ok and what is not None:
            msg = getattr(thrown, "message", str(thrown))
            if isinstance(what, str):
                ok = what in msg
            elif isinstance(what, type):
                ok = isinstance(thrown, what)
        self._check(ok, f"to throw {what!r}")


setattr(_Expect, "not", property(lambda self: _Expect(self.v, not self.negate)))


class _OutOfTime(BaseException):
    pass


def bun_test_module(results, select=None, budget_s=None):
    """describe/test/expect: each test runs when it is declared and appends (name, error or None) to
    `results`. `select`: the ordinals of the tests to run (the others are listed as "not selected");
    `budget_s`: a test still running after that many seconds is stopped and listed as out of time."""
    import signal
    prefix = []
    count = [0]

    def _alarm(*_):
        raise _OutOfTime()

    def describe(name, fn=None, *_):
        prefix.append(str(name))
        try:
            fn()
        finally:
            prefix.pop()

    def test(name, fn=None, *_):
        full = " > ".join(prefix + [str(name)])
        k = count[0]
        count[0] += 1
        if select is not None and k not in select:
            results.append((full, "not selected"))
            return
        if budget_s:
            signal.signal(signal.SIGALRM, _alarm)
            signal.alarm(int(budget_s))
        try:
            fn()
            results.append((full, None))
        except _OutOfTime:
            results.append((full, f"out of time: still running after {budget_s} s"))
        except Exception as e:  # noqa: BLE001 - record the failure and go on
            results.append((full, f"{type(e).__name__}: {e}"))
        finally:
            if budget_s:
                signal.alarm(0)

    def skip(name, fn=None, *_):
        results.append((" > ".join(prefix + [str(name)]), "skipped"))

    setattr(test, "skip", skip)
    setattr(test, "todo", skip)
    expect_obj = lambda v=None, *_: _Expect(v)  # noqa: E731
    return {"describe": describe, "test": test, "it": test, "expect": expect_obj}
