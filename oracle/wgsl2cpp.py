"""Translate the reference's attention WGSL shaders (with ARGMAX, which advances the meta
buffer, and the MatMulNBits GEMV / GEMM around the path) into C++ for host execution.

TEST INFRASTRUCTURE ONLY.  The reference keeps its GPU code as WGSL template strings inside
JavaScript modules (src/scripts/lfm-engine/kernels.js, vision-kernels.js) and runs them
through WebGPU, which does not exist on this machine.  This script reads those modules from
the reference checkout, extracts the shaders named on the command line, and rewrites the WGSL
subset they use into C++20 (one coroutine per invocation, see oracle/wgsl_rt.h).  Output goes
to oracle/_ref/ only; it is generated at build time and never committed.

The translation is purely mechanical (declarations -> globals, `let`/`var` -> `auto`,
abstract float literals -> f32 literals, builtins -> wgsl:: functions, workgroupBarrier() ->
co_await, return -> co_return); the statements, their order and every constant stay as
written in the reference.

Usage: python oracle/wgsl2cpp.py <reference_root> <out.cpp>
"""
from __future__ import annotations

import re
import sys
from pathlib import Path

# (module relative to the reference root, exported shader constant)
SHADERS = [
    ("src/scripts/lfm-engine/kernels.js", "QK_PREP"),
    ("src/scripts/lfm-engine/kernels.js", "ATTN"),
    ("src/scripts/lfm-engine/vision-kernels.js", "VISION_ATTN"),
    ("src/scripts/lfm-engine/kernels.js", "ARGMAX"),
    ("src/scripts/lfm-engine/kernels.js", "GEMV"),
    ("src/scripts/lfm-engine/kernels.js", "GEMM"),
]

TYPES = {"f32": "float", "f16": "wgsl::h16", "u32": "uint32_t", "i32": "int32_t"}

FLOAT_LIT = re.compile(r"(?<![\w.])(\d+\.\d*(?:[eE][+-]?\d+)?|\d+[eE][+-]?\d+|\.\d+(?:[eE][+-]?\d+)?)(?![\w.])")


def extract(src: str, name: str) -> str:
    m = re.search(r"export const " + name + r" = `\$\{HEAD\}(.*?)`;", src, re.S)
    if not m:
        raise SystemExit(f"shader {name} not found")
    body = m.group(1)

    # snippets the shader interpolates (e.g. the GEMV's ${ZP_FN}) are module constants
    def snippet(sm):
        c = re.search(r"const " + sm.group(1) + r" = `(.*?)`;", src, re.S)
        if not c or "${" in c.group(1):
            raise SystemExit(f"shader {name}: snippet {sm.group(1)} not found or nested")
        return c.group(1)

    body = re.sub(r"\$\{(\w+)\}", snippet, body)
    return body


def translate_expr(line: str) -> str:
    line = FLOAT_LIT.sub(lambda m: m.group(1) + "f", line)
    line = re.sub(r"\bworkgroupBarrier\(\);", "co_await wgsl::Barrier{};", line)
    line = re.sub(r"\breturn;", "co_return;", line)
    line = re.sub(r"\blet\s+(\w+)\s*=", r"const auto \1 =", line)
    line = re.sub(r"\bvar\s+(\w+)\s*:\s*(\w+)\s*=", lambda m: f"{TYPES[m.group(2)]} {m.group(1)} =", line)
    line = re.sub(r"\bvar\s+(\w+)\s*=", r"auto \1 =", line)
    line = re.sub(r"\barray<vec4<f32>,\s*4>\(", "wgsl::array4v(", line)
    line = re.sub(r"\bvec4<f32>\(", "wgsl::vec4f(", line)
    line = re.sub(r"\b(f32|f16|u32)\(", r"wgsl::\1(", line)
    line = re.sub(r"\bexp\(", "wgsl::exp_(", line)
    line = re.sub(r"\binverseSqrt\(", "wgsl::inverseSqrt(", line)
    line = re.sub(r"\bmax\(", "wgsl::max_(", line)
    line = re.sub(r"\bmin\(", "wgsl::min_(", line)
    return line


def translate(name: str, wgsl: str) -> str:
    ns = f"sh_{name}"
    overrides, bindings, wgvars = [], {}, []
    wg_size = None
    params = {}
    body: list[str] = []
    helpers: list[str] = []
    in_main = False
    in_fn = False
    for raw in wgsl.splitlines():
        line = raw.strip()
        if not line or line.startswith("enable "):
            continue
        if in_main:
            body.append(translate_expr(raw))
            continue
        if in_fn:  # a helper function's body, up to its closing brace at column 0
            helpers.append(translate_expr(raw))
            if raw.startswith("}"):
                in_fn = False
            continue
        if m := re.match(r"fn (\w+)\((.*)\)\s*->\s*(\w+)\s*\{", line):
            if m.group(1) != "main":
                args = []
                for a in m.group(2).split(","):
                    am = re.match(r"\s*(\w+)\s*:\s*(\w+)\s*$", a)
                    if not am:
                        raise SystemExit(f"{name}: unsupported helper parameter {a!r}")
                    args.append(f"{TYPES[am.group(2)]} {am.group(1)}")
                helpers.append(f"static {TYPES[m.group(3)]} {m.group(1)}({', '.join(args)}) {{")
                in_fn = True
                continue
        if m := re.match(r"override (\w+): (\w+) = ([^;]+);", line):
            overrides.append((m.group(1), TYPES[m.group(2)], translate_expr(m.group(3))))
            continue
        if m := re.match(r"override (\w+): (\w+);", line):  # no default: set by the runner
            overrides.append((m.group(1), TYPES[m.group(2)], "0"))
            continue
        if m := re.match(r"@group\(0\) @binding\((\d+)\) var<storage, (\w+)> (\w+): array<(\w+)>;", line):
            bindings[int(m.group(1))] = (m.group(3), TYPES[m.group(4)], m.group(2))
            continue
        if m := re.match(r"var<workgroup> (\w+): array<(\w+), (\w+)>;", line):
            wgvars.append((m.group(1), TYPES[m.group(2)], m.group(3)))
            continue
        if m := re.match(r"@compute @workgroup_size\((\w+)\)", line):
            wg_size = m.group(1)
            line = line[m.end():].strip()
            if not line:
                continue
        if m := re.match(r"fn main\((.*)\)\s*\{", line):
            for p in m.group(1).split(","):
                pm = re.match(r"\s*@builtin\((\w+)\)\s*(\w+)\s*:", p)
                if not pm:
                    raise SystemExit(f"{name}: unsupported parameter {p!r}")
                params[pm.group(1)] = pm.group(2)
            in_main = True
            continue
        raise SystemExit(f"{name}: unsupported declaration {line!r}")
    if wg_size is None or not in_main:
        raise SystemExit(f"{name}: no entry point")
    # The last line of the body is the closing brace of main.
    while body and not body[-1].strip():
        body.pop()
    if body[-1].strip() != "}":
        raise SystemExit(f"{name}: unexpected end of main")
    body = body[:-1]

    out = [f"namespace {ns} {{"]
    for oname, otype, odef in overrides:
        out.append(f"static {otype} {oname} = {odef};")
    for idx in sorted(bindings):
        bname, btype, access = bindings[idx]
        out.append(f"static {btype}* {bname} = nullptr;  // binding {idx} ({access})")
    for vname, vtype, vlen in wgvars:
        out.append(f"static thread_local {vtype} {vname}[{vlen}];")
    out.extend(helpers)
    wid = params.get("workgroup_id", "wid_unused")
    lid = params.get("local_invocation_index", "lid_unused")
    out.append(f"static wgsl::Task main_(wgsl::uvec3 {wid}, uint32_t {lid}) {{")
    out.extend(body)
    out.append("  co_return;")
    out.append("}")
    out.append("static void reset_wg() {")
    for vname, _, _ in wgvars:
        out.append(f"  std::memset({vname}, 0, sizeof({vname}));")
    out.append("}")
    out.append(f"}}  // namespace {ns}")
    # Runner: bindings in binding order, overrides in declaration order (as doubles).
    out.append(f'extern "C" int ref_{name}(void* const* bindings, const double* overrides,')
    out.append("                          uint32_t gx, uint32_t gy, uint32_t gz) {")
    for i, idx in enumerate(sorted(bindings)):
        bname, btype, _ = bindings[idx]
        out.append(f"  {ns}::{bname} = static_cast<{btype}*>(bindings[{i}]);")
    for i, (oname, otype, _) in enumerate(overrides):
        out.append(f"  if (overrides) {ns}::{oname} = static_cast<{otype}>(overrides[{i}]);")
    size_expr = wg_size if not wg_size.isidentifier() else f"{ns}::{wg_size}"
    out.append(f"  return wgsl::dispatch(gx, gy, gz, uint32_t({size_expr}),")
    out.append(f"      [](wgsl::uvec3 w, uint32_t t) {{ return {ns}::main_(w, t); }}, {ns}::reset_wg);")
    out.append("}")
    out.append(f'extern "C" int ref_{name}_nbindings() {{ return {len(bindings)}; }}')
    out.append(f'extern "C" int ref_{name}_noverrides() {{ return {len(overrides)}; }}')
    return "\n".join(out) + "\n"


def main() -> None:
    root, dst = Path(sys.argv[1]), Path(sys.argv[2])
    parts = [
        "// GENERATED by oracle/wgsl2cpp.py from the reference's WGSL shaders. Do not commit.\n",
        '#include "wgsl_rt.h"\n',
        "#pragma GCC diagnostic ignored \"-Wunused-variable\"\n",
    ]
    for module, name in SHADERS:
        parts.append(f"// ---- {name} from {module}\n")
        parts.append(translate(name, extract((root / module).read_text(), name)))
    dst.parent.mkdir(parents=True, exist_ok=True)
    dst.write_text("".join(parts))


if __name__ == "__main__":
    main()
