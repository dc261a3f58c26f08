"""WGSL -> C++ source translator for the reference's compute shaders - TEST INFRASTRUCTURE.

The reference (dparnell/sense-nova-server) runs its hot path as WGSL compute shaders
through wgpu; neither wgpu, a graphics stack nor Rust exists on these machines. This
script runs those shaders on the host cores instead: it translates each shader module,
read from the reference tree at build time, into C++ against oracle/wgsl_rt.h and
compiles it into oracle/_ref/libwgslref.so. The translation is mechanical (declarations,
literals, builtins); every expression keeps the shader's own operands and order, so the
library computes what the shader source says, in f32, with host libm transcendentals.
The generated C++ and the library stay in oracle/_ref/ (git-ignored): no reference
source is copied into the repository.

Modules (the splices of src/gpu.rs:367-375 and src/vision.rs:111):
  matmul_q8 / matmul_q4  src/shaders/matmul.wgsl with //QUANT_FNS// replaced by
                         gpu.rs's Q8_FNS / Q4_FNS (gpu.rs:236-308)
  layers, attention, linear, vision   src/shaders/<name>.wgsl as is

Usage: python oracle/wgsl2cpp.py [--ref /root/reference] [--out oracle/_ref]
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEFAULT_REF = Path(os.environ.get("SNL_REFERENCE", "/root/reference"))
OUT = HERE / "_ref"
LIB = OUT / "libwgslref.so"
MODULES = ["matmul_q8", "matmul_q4", "layers", "attention", "linear", "vision"]

BUILTINS = {"exp", "log", "pow", "sin", "cos", "tanh", "sqrt", "inverseSqrt", "abs", "max", "min", "clamp",
            "select", "dot", "pack2x16float", "unpack2x16float", "workgroupBarrier", "storageBarrier"}
BUILTIN_VARS = {"global_invocation_id", "local_invocation_id", "local_invocation_index", "workgroup_id",
                "num_workgroups"}
CPP_RESERVED = {
    "auto", "char", "class", "default", "delete", "double", "do", "enum", "explicit", "export", "extern", "float",
    "friend", "goto", "inline", "int", "long", "mutable", "namespace", "new", "operator", "private", "protected",
    "public", "register", "short", "signed", "sizeof", "static", "template", "this", "throw", "try", "catch",
    "typedef", "typename", "union", "unsigned", "using", "virtual", "volatile", "and", "or", "not", "xor",
    "bitand", "bitor", "compl", "asm", "wgsl", "std", "array", "vec2", "vec3", "vec4", "mat4x4", "Buf",
    "Builtins", "dispatch", "zero_wg", "bi", "NAN", "INFINITY", "assert", "errno"}
TYPE_HEADS = {"vec2", "vec3", "vec4", "mat4x4", "array", "ptr", "atomic"}

TOKEN_RE = re.compile(r"""
    (?P<ws>\s+)
  | (?P<comment>//[^\n]*|/\*.*?\*/)
  | (?P<num>0[xX][0-9a-fA-F]+[iu]?|(?:\d+\.\d*|\.\d+|\d+)(?:[eE][+-]?\d+)?[fhiu]?)
  | (?P<id>[A-Za-z_][A-Za-z0-9_]*)
  | (?P<op><<=|>>=|->|<<|>>|<=|>=|==|!=|&&|\|\||\+=|-=|\*=|/=|%=|&=|\|=|\^=|\+\+|--|[{}()\[\];:,.<>=+\-*/%&|^!~@?])
""", re.X | re.S)


def tokenize(src: str) -> list[str]:
    out, i = [], 0
    while i < len(src):
        m = TOKEN_RE.match(src, i)
        if not m:
            raise SyntaxError(f"wgsl2cpp: cannot tokenize at {src[i:i + 40]!r}")
        i = m.end()
        if m.lastgroup in ("ws", "comment"):
            continue
        out.append(m.group())
    return out


def literal(tok: str) -> str:
    """A WGSL numeric literal as a C++ literal of the same type (f32 for floats)."""
    if tok.lower().startswith("0x"):
        return tok[:-1] if tok.endswith("i") else tok
    is_float = any(c in tok for c in ".eE") or tok.endswith(("f", "h"))
    if is_float:
        body = tok.rstrip("fh")
        if "." not in body and "e" not in body.lower():
            body += ".0"
        return body + "f"
    return tok[:-1] if tok.endswith("i") else tok


class Module:
    def __init__(self, name: str, src: str):
        self.name = name
        self.t = tokenize(src)
        self.i = 0
        self.structs: list[str] = []   # structs and consts, in source order
        self.bindings: list[tuple[int, str, str, str]] = []  # (binding, name, kind, ctype)
        self.wg_vars: list[tuple[str, str]] = []
        self.protos: list[str] = []
        self.bodies: list[str] = []
        self.entries: list[tuple[str, tuple[int, int, int]]] = []
        self.user_fns = {self.t[k + 1] for k in range(len(self.t) - 1) if self.t[k] == "fn"}

    # -- token helpers --
    def peek(self, k: int = 0) -> str:
        return self.t[self.i + k] if self.i + k < len(self.t) else ""

    def take(self, expect: str | None = None) -> str:
        tok = self.peek()
        if expect is not None and tok != expect:
            raise SyntaxError(f"{self.name}: expected {expect!r}, got {tok!r} near {' '.join(self.t[self.i - 5:self.i + 5])}")
        self.i += 1
        return tok

    def ident(self, tok: str) -> str:
        if tok in self.user_fns:
            return "u_" + tok
        return tok + "_" if tok in CPP_RESERVED else tok

    def split_gt(self) -> None:
        """Split a '>>' / '>=' / '>>=' token so a template close can be taken alone."""
        tok = self.peek()
        if tok in (">>", ">=", ">>="):
            self.t[self.i:self.i + 1] = [">", tok[1:]]

    # -- types --
    def type_(self) -> str:
        head = self.take()
        if head in ("vec2", "vec3", "vec4", "mat4x4"):
            self.take("<")
            inner = self.type_()
            self.split_gt()
            self.take(">")
            return f"{head}<{inner}>"
        if head in ("vec2f", "vec3f", "vec4f", "vec2u", "vec3u", "vec4u", "vec2i", "vec3i", "vec4i"):
            return f"{head[:4]}<{ {'f': 'f32', 'u': 'u32', 'i': 'i32'}[head[4]] }>"
        if head == "array":
            self.take("<")
            inner = self.type_()
            if self.peek() == ",":
                self.take(",")
                n = self.expr_until({">"}, template=True)
                self.split_gt()
                self.take(">")
                return f"array<{inner}, {n}>"
            self.split_gt()
            self.take(">")
            return f"RUNTIME<{inner}>"
        if head == "ptr":
            self.take("<")
            self.take()  # address space
            self.take(",")
            inner = self.type_()
            if self.peek() == ",":
                self.take(",")
                self.take()
            self.split_gt()
            self.take(">")
            return f"{inner}*"
        if head in ("atomic",):
            raise SyntaxError(f"{self.name}: atomics are not supported")
        return self.ident(head)

    # -- expressions (token rewrite until a stop token at depth 0) --
    def expr_until(self, stops: set[str], template: bool = False) -> str:
        out: list[str] = []
        depth = 0
        while True:
            tok = self.peek()
            if tok == "":
                raise SyntaxError(f"{self.name}: unexpected end of source")
            if depth == 0 and (tok in stops or (template and tok in (">>", ">=", ">>="))):
                return " ".join(out)
            if tok in ("(", "["):
                depth += 1
            elif tok in (")", "]"):
                depth -= 1
                if depth < 0:
                    return " ".join(out)
            if tok in TYPE_HEADS or tok in ("vec2f", "vec3f", "vec4f", "vec2u", "vec3u", "vec4u", "vec2i",
                                            "vec3i", "vec4i"):
                ty = self.type_()
                out.append(ty)
                continue
            if tok == "bitcast":
                self.take()
                self.take("<")
                ty = self.type_()
                self.split_gt()
                self.take(">")
                out.append(f"wgsl_bitcast<{ty}>")
                continue
            self.take()
            if tok[0].isdigit() or (tok[0] == "." and len(tok) > 1):
                out.append(literal(tok))
            elif tok[0].isalpha() or tok[0] == "_":
                if out and out[-1] == ".":  # member access: field or vector component
                    out.append(tok + "_" if tok in CPP_RESERVED else tok)
                elif tok in BUILTINS and self.peek() == "(":
                    out.append("W_" + tok)
                else:
                    out.append(self.ident(tok))
            else:
                out.append(tok)

    # -- statements --
    def block(self) -> str:
        self.take("{")
        lines = []
        while self.peek() != "}":
            lines.append(self.statement())
        self.take("}")
        return "{\n" + "\n".join(lines) + "\n}"

    def decl(self, kind: str) -> str:
        """`let`/`var` declaration up to (not including) ';'."""
        name = self.ident(self.take())
        ty = None
        if self.peek() == ":":
            self.take(":")
            ty = self.type_()
        if self.peek() == "=":
            self.take("=")
            e = self.expr_until({";"})
            if ty is None:
                return f"{'const ' if kind == 'let' else ''}auto {name} = {e}"
            return f"{'const ' if kind == 'let' else ''}{ty} {name} = {e}"
        if ty is None:
            raise SyntaxError(f"{self.name}: declaration of {name} without type or value")
        return f"{ty} {name}{{}}"

    def statement(self) -> str:
        tok = self.peek()
        if tok == "{":
            return self.block()
        if tok in ("let", "var", "const"):
            self.take()
            s = self.decl("let" if tok != "var" else "var")
            self.take(";")
            return s + ";"
        if tok == "if":
            self.take()
            cond = self.expr_until({"{"})
            s = f"if ({cond}) " + self.block()
            while self.peek() == "else":
                self.take()
                if self.peek() == "if":
                    s += " else " + self.statement()
                    break
                s += " else " + self.block()
            return s
        if tok == "for":
            self.take()
            self.take("(")
            init = ""
            if self.peek() in ("var", "let"):
                kind = self.take()
                init = self.decl(kind)
            elif self.peek() != ";":
                init = self.expr_until({";"})
            self.take(";")
            cond = self.expr_until({";"})
            self.take(";")
            upd = self.expr_until({")"})
            self.take(")")
            return f"for ({init}; {cond}; {upd}) " + self.block()
        if tok == "while":
            self.take()
            cond = self.expr_until({"{"})
            return f"while ({cond}) " + self.block()
        if tok == "loop":
            self.take()
            body = self.block()
            if "continuing" in body:
                raise SyntaxError(f"{self.name}: loop continuing blocks are not supported")
            return "for (;;) " + body
        if tok in ("break", "continue"):
            self.take()
            self.take(";")
            return tok + ";"
        if tok == "return":
            self.take()
            if self.peek() == ";":
                self.take()
                return "return;"
            e = self.expr_until({";"})
            self.take(";")
            return f"return {e};"
        if tok == "switch":
            raise SyntaxError(f"{self.name}: switch is not supported")
        e = self.expr_until({";"})
        self.take(";")
        return e + ";"

    # -- module level --
    def attrs(self) -> dict[str, list[str]]:
        a: dict[str, list[str]] = {}
        while self.peek() == "@":
            self.take("@")
            name = self.take()
            args: list[str] = []
            if self.peek() == "(":
                self.take("(")
                while self.peek() != ")":
                    args.append(self.expr_until({",", ")"}))
                    if self.peek() == ",":
                        self.take(",")
                self.take(")")
            a[name] = args
        return a

    def translate(self) -> None:
        while self.i < len(self.t):
            at = self.attrs()
            tok = self.take()
            if tok == "struct":
                name = self.ident(self.take())
                self.take("{")
                fields = []
                while self.peek() != "}":
                    self.attrs()
                    f = self.ident(self.take())
                    self.take(":")
                    fields.append(f"  {self.type_()} {f};")
                    if self.peek() == ",":
                        self.take(",")
                self.take("}")
                if self.peek() == ";":
                    self.take(";")
                self.structs.append(f"struct {name} {{\n" + "\n".join(fields) + "\n};")
            elif tok == "const":
                name = self.ident(self.take())
                ty = "auto"
                if self.peek() == ":":
                    self.take(":")
                    ty = self.type_()
                self.take("=")
                e = self.expr_until({";"})
                self.take(";")
                self.structs.append(f"constexpr {ty} {name} = {e};")
            elif tok == "var":
                space = []
                if self.peek() == "<":
                    self.take("<")
                    while self.peek() != ">":
                        space.append(self.take())
                    self.take(">")
                name = self.ident(self.take())
                self.take(":")
                ty = self.type_()
                self.take(";")
                sp = space[0] if space else "private"
                if sp == "workgroup":
                    self.wg_vars.append((name, ty))
                elif sp in ("uniform", "storage"):
                    b = int(at["binding"][0].rstrip("u"))
                    if sp == "uniform":
                        self.bindings.append((b, name, "uniform", ty))
                    else:
                        inner = ty[len("RUNTIME<"):-1] if ty.startswith("RUNTIME<") else None
                        if inner is None:
                            raise SyntaxError(f"{self.name}: fixed-size storage binding {name}")
                        self.bindings.append((b, name, "storage", inner))
                else:
                    raise SyntaxError(f"{self.name}: module-scope var<{sp}> {name}")
            elif tok == "fn":
                self.function(at)
            elif tok in ("enable", "requires", "diagnostic"):
                while self.take() != ";":
                    pass
            else:
                raise SyntaxError(f"{self.name}: unexpected {tok!r} at module scope")

    def function(self, at: dict[str, list[str]]) -> None:
        raw = self.take()
        name = self.ident(raw)
        self.take("(")
        params, builtins = [], []
        while self.peek() != ")":
            pa = self.attrs()
            pn = self.ident(self.take())
            self.take(":")
            pt = self.type_()
            if "builtin" in pa:
                bname = pa["builtin"][0]
                if bname not in BUILTIN_VARS:
                    raise SyntaxError(f"{self.name}: builtin {bname}")
                builtins.append(f"const {pt} {pn} = bi.{bname};")
            else:
                params.append(f"{pt} {pn}")
            if self.peek() == ",":
                self.take(",")
        self.take(")")
        ret = "void"
        if self.peek() == "->":
            self.take("->")
            self.attrs()
            ret = self.type_()
        body = self.block()
        if "compute" in at:
            ws = [int(v.rstrip("u")) for v in at["workgroup_size"]] + [1, 1]
            self.entries.append((raw, (ws[0], ws[1], ws[2])))
            self.bodies.append(f"static void e_{raw}(const Builtins& bi) {{\n" + "\n".join(builtins) + "\n"
                               + body[1:])
        else:
            sig = f"static {ret} {name}({', '.join(params)})"
            self.protos.append(sig + ";")
            self.bodies.append(sig + " " + body)

    def cpp(self) -> str:
        ns = f"wr_{self.name}"
        out = ['#include "wgsl_rt.h"', f"namespace {ns} {{", "using namespace wgsl;",
               "template <class T, class F> T wgsl_bitcast(F v) { static_assert(sizeof(T) == sizeof(F)); T r; "
               "std::memcpy(&r, &v, sizeof(T)); return r; }"]
        out += self.structs
        for b, n, kind, ty in self.bindings:
            out.append(f"static {ty} {n};" if kind == "uniform" else f"static Buf<{ty}> {n};")
        for n, ty in self.wg_vars:  # one copy per host thread: each thread runs its own workgroup
            out.append(f"static thread_local {ty} {n};")
        out.append("static void zero_wg() {" + " ".join(f"{n} = {ty}{{}};" for n, ty in self.wg_vars) + "}")
        out += self.protos
        out += self.bodies
        # binding setter and dispatcher
        out.append("static int bind(int wr_slot, void* wr_ptr, uint64_t wr_bytes) {")
        out.append("  switch (wr_slot) {")
        for b, n, kind, ty in self.bindings:
            if kind == "uniform":
                out.append(f"    case {b}: if (wr_bytes < sizeof({ty})) return -2; std::memcpy(&{n}, wr_ptr, sizeof({ty})); return 0;")
            else:
                out.append(f"    case {b}: {n}.p = static_cast<{ty}*>(wr_ptr); {n}.n = wr_bytes / sizeof({ty}); return 0;")
        out.append("  }\n  return -1;\n}")
        out.append("}  // namespace " + ns)
        out.append(f'extern "C" int64_t {ns}_dispatch(const char* entry, uint32_t gx, uint32_t gy, uint32_t gz, '
                   "int nb, const int* binding, void* const* ptr, const uint64_t* bytes) {")
        out.append(f"  using namespace {ns};")
        out.append("  for (int k = 0; k < nb; k++) if (bind(binding[k], ptr[k], bytes[k])) return -2 - k;")
        for raw, (x, y, z) in self.entries:
            out.append(f'  if (!std::strcmp(entry, "{raw}")) return (int64_t)dispatch(e_{raw}, zero_wg, gx, gy, gz, '
                       f"{x}, {y}, {z});")
        out.append("  return -1;\n}")
        out.append(f'extern "C" const char* {ns}_entries() {{ return "'
                   + ",".join(f"{r}:{x}x{y}x{z}" for r, (x, y, z) in self.entries) + '"; }')
        return "\n".join(out) + "\n"


def rust_raw_string(src: str, const: str) -> str:
    m = re.search(r"const\s+" + const + r'\s*:\s*&str\s*=\s*r#"(.*?)"#;', src, re.S)
    if not m:
        raise SyntaxError(f"gpu.rs: {const} not found")
    return m.group(1)


def module_sources(ref: Path) -> dict[str, str]:
    sh = ref / "src" / "shaders"
    gpu = (ref / "src" / "gpu.rs").read_text()
    mm = (sh / "matmul.wgsl").read_text()
    srcs = {
        "matmul_q8": mm.replace("//QUANT_FNS//", rust_raw_string(gpu, "Q8_FNS")),
        "matmul_q4": mm.replace("//QUANT_FNS//", rust_raw_string(gpu, "Q4_FNS")),
    }
    for n in ("layers", "attention", "linear", "vision"):
        srcs[n] = (sh / f"{n}.wgsl").read_text()
    return srcs


def build(ref: Path = DEFAULT_REF, out: Path = OUT, force: bool = False) -> Path | None:
    """Translate and compile the reference's shaders. None when the reference is absent."""
    if not (ref / "src" / "shaders").is_dir():
        return None
    lib = out / "libwgslref.so"
    deps = [HERE / "wgsl_rt.h", Path(__file__)] + sorted((ref / "src" / "shaders").glob("*.wgsl")) + [ref / "src" / "gpu.rs"]
    if not force and lib.exists() and all(lib.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return lib
    return compile_modules(module_sources(ref), out, lib.name)


def compile_modules(srcs: dict[str, str], out: Path, lib_name: str) -> Path:
    """Translate WGSL modules {name: source} and link them into out/lib_name; module
    `name` exports wr_<name>_dispatch and wr_<name>_entries."""
    out.mkdir(parents=True, exist_ok=True)
    cpps = []
    for name, src in srcs.items():
        m = Module(name, src)
        m.translate()
        p = out / f"wgsl_{name}.cpp"
        p.write_text(m.cpp())
        cpps.append(p)
    lib = out / lib_name
    cxx = os.environ.get("SNL_CXX") or shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++20", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread",
           "-I", str(HERE), *map(str, cpps), "-o", str(lib)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"wgsl2cpp: compile failed:\n{r.stderr[-6000:]}")
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=Path, default=DEFAULT_REF)
    ap.add_argument("--out", type=Path, default=OUT)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    lib = build(a.ref, a.out, a.force)
    print(lib if lib else "reference tree absent: nothing built", file=sys.stderr)


if __name__ == "__main__":
    main()
