"""The Rust binding (qora-llm-4b_b200/rust) against the C header, on the CPU.

No Rust toolchain exists on these machines, so the crates cannot be built;
this test keeps them from drifting from include/qora_mixer.h instead.  It
parses both and checks that every header function is declared in the sys
crate's extern block with the same name, argument count, argument types
(integer widths, pointer constness and depth) and return type; that every
struct has the same fields in the same order with the same types; that the
QM_* constants have the same values; and that the safe wrapper only calls
functions the sys crate declares.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qora_mixer.h")
RUST = os.path.join(ROOT, "qora-llm-4b_b200", "rust")
SYS = os.path.join(RUST, "qora-mixer-sys", "src", "lib.rs")
SAFE = os.path.join(RUST, "qora-mixer", "src", "lib.rs")

C_BASE = {"int": "i32", "int64_t": "i64", "size_t": "usize", "float": "f32", "double": "f64",
          "uint16_t": "u16", "char": "i8", "unsigned char": "u8", "void": "void"}
R_BASE = {"c_int": "i32", "i32": "i32", "i64": "i64", "usize": "usize", "f32": "f32", "f64": "f64",
          "u16": "u16", "c_char": "i8", "c_uchar": "u8", "u8": "u8", "c_void": "void", "u32": "u32"}


def _strip_c(src):
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.sub(r"//[^\n]*", "", src)


def c_type(decl, has_name=True):
    """('ptr', pointee_const, inner) trees for a C declarator (name dropped)."""
    toks = re.findall(r"\*|[A-Za-z_]\w*", decl)
    if has_name and toks and toks[-1] not in ("*", "const") and len(toks) > 1:
        toks = toks[:-1]
    base_const = False
    base = []
    i = 0
    while i < len(toks) and toks[i] != "*":
        if toks[i] == "const":
            base_const = True
        else:
            base.append(toks[i])
        i += 1
    name = " ".join(base)
    cur = C_BASE.get(name, name)
    cur_const = base_const
    while i < len(toks):
        if toks[i] == "*":
            cur = ("ptr", cur_const, cur)
            cur_const = False
        elif toks[i] == "const":
            cur_const = True
        i += 1
    return cur


def r_type(t):
    t = " ".join(t.split())
    m = re.match(r"^\*(const|mut)\s+(.*)$", t)
    if m:
        return ("ptr", m.group(1) == "const", r_type(m.group(2)))
    t = t.split("::")[-1]
    return R_BASE.get(t, t)


def header_functions():
    src = _strip_c(open(HEADER).read())
    src = re.sub(r"^\s*#.*$", "", src, flags=re.M)
    out = {}
    for stmt in src.split(";"):
        st = " ".join(stmt.split()).split("}")[-1].strip()
        m = re.match(r"^((?:const\s+)?[A-Za-z_]\w*\s*\**)\s*(qm_\w+)\s*\((.*)\)$", st)
        if not m:
            continue
        args = [a.strip() for a in m.group(3).split(",") if a.strip() and a.strip() != "void"]
        out[m.group(2)] = (c_type(m.group(1), has_name=False), [c_type(a) for a in args])
    return out


def header_structs():
    src = _strip_c(open(HEADER).read())
    out = {}
    for m in re.finditer(r"typedef struct (qm_\w+) \{(.*?)\}\s*\1\s*;", src, flags=re.S):
        fields = []
        for line in m.group(2).split(";"):
            line = " ".join(line.split())
            if not line:
                continue
            # "int world, rank" declares two fields of one type
            head, *rest = [x.strip() for x in line.split(",")]
            t = c_type(head)
            fields.append((head.split()[-1].lstrip("*"), t))
            for r in rest:
                fields.append((r, t))
        out[m.group(1)] = fields
    return out


def header_defines():
    src = open(HEADER).read()
    out = {}
    for m in re.finditer(r"^#define (QM_\w+)\s+\(?(\d+)u?(?:\s*<<\s*(\d+))?\)?", src, flags=re.M):
        v = int(m.group(2))
        if m.group(3):
            v <<= int(m.group(3))
        out[m.group(1)] = v
    return out


def rust_sys():
    src = re.sub(r"//[^\n]*", "", open(SYS).read())
    block = src[src.index('extern "C" {'):]
    fns = {}
    for m in re.finditer(r"pub fn (qm_\w+)\s*\((.*?)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        args = [a.strip() for a in m.group(2).split(",") if a.strip()]
        types = [r_type(a.split(":", 1)[1]) for a in args]
        ret = r_type(m.group(3)) if m.group(3) else "void"
        fns[m.group(1)] = (ret, types)
    structs = {}
    for m in re.finditer(r"pub struct (qm_\w+)\s*\{(.*?)\}", src, flags=re.S):
        body = m.group(2)
        if "_private" in body:
            continue
        fields = []
        for f in body.split(","):
            f = f.strip()
            if not f:
                continue
            nm, ty = f.split(":", 1)
            fields.append((nm.replace("pub", "").strip(), r_type(ty)))
        structs[m.group(1)] = fields
    consts = {}
    for m in re.finditer(r"pub const (QM_\w+):\s*\w+\s*=\s*(\d+)(?:u32)?(?:\s*<<\s*(\d+))?;", src):
        v = int(m.group(2))
        if m.group(3):
            v <<= int(m.group(3))
        consts[m.group(1)] = v
    opaque = set(re.findall(r"pub struct (qm_\w+)\s*\{\s*_private", src))
    return fns, structs, consts, opaque


def test_every_header_function_is_declared_alike():
    hf = header_functions()
    rf, _, _, _ = rust_sys()
    assert len(hf) >= 60
    missing = sorted(set(hf) - set(rf))
    extra = sorted(set(rf) - set(hf))
    assert not missing, f"declared in the header, missing in the Rust binding: {missing}"
    assert not extra, f"declared in the Rust binding, absent from the header: {extra}"
    for name, (cret, cargs) in hf.items():
        rret, rargs = rf[name]
        assert len(cargs) == len(rargs), f"{name}: {len(cargs)} C arguments, {len(rargs)} Rust"
        for i, (ca, ra) in enumerate(zip(cargs, rargs)):
            assert ca == ra, f"{name} argument {i}: C {ca} vs Rust {ra}"
        assert cret == rret, f"{name} returns C {cret} vs Rust {rret}"


def test_structs_have_the_same_fields():
    hs = header_structs()
    _, rs, _, opaque = rust_sys()
    assert set(hs) == {"qm_shape", "qm_dn_params", "qm_gqa_params", "qm_weight", "qm_shard"}
    for name, fields in hs.items():
        assert name in rs, name
        assert fields == rs[name], f"{name}: C {fields} vs Rust {rs[name]}"
    assert {"qm_ctx", "qm_dn_state", "qm_kv", "qm_comm"} <= opaque


def test_constants_match():
    hd = header_defines()
    _, _, rc, _ = rust_sys()
    assert "QM_E_CAPTURE" in hd and "QM_W_Q4_ROWS" in hd and "QM_NOALLOC_SCRATCH_BYTES" in hd
    for k, v in hd.items():
        assert rc.get(k) == v, f"{k}: header {v}, Rust {rc.get(k)}"


def test_weight_kinds_are_the_four_formats():
    hd = header_defines()
    assert [hd[k] for k in ("QM_W_F16", "QM_W_Q4", "QM_W_F16_ROWS", "QM_W_Q4_ROWS")] == [0, 1, 2, 3]


def test_safe_wrapper_calls_only_declared_functions():
    rf, _, _, _ = rust_sys()
    used = set(re.findall(r"sys::(qm_\w+)\s*\(", open(SAFE).read()))
    assert used, "the wrapper calls nothing"
    assert used <= set(rf), sorted(used - set(rf))
    # every handle the wrapper owns is destroyed in Drop
    src = open(SAFE).read()
    for kind in ("qm_ctx_destroy", "qm_dn_state_destroy", "qm_kv_destroy"):
        assert kind in used


def test_parser_reads_pointer_forms():
    assert c_type("float* const* ys") == ("ptr", True, ("ptr", False, "f32"))
    assert r_type("*const *mut f32") == ("ptr", True, ("ptr", False, "f32"))
    assert c_type("const unsigned char* id") == ("ptr", True, "u8")
    assert c_type("qm_ctx** out") == ("ptr", False, ("ptr", False, "qm_ctx"))
    assert c_type("int64_t seq_len") == "i64"
