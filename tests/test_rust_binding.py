"""include/cuda.rs (the Rust host's `src/cuda.rs`) declares every entry
point of include/molten_cuda.h with matching parameters: same names, same
count and order, and each C type mapped to its Rust FFI type (pointer
constness included); the structs and constants agree too. rustc is not in
this image, so the check is textual."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

C_BASE = {"int": "c_int", "size_t": "usize", "float": "f32", "uint32_t": "u32",
          "uint64_t": "u64", "int32_t": "i32", "unsigned long long": "u64", "void": "c_void",
          "uint16_t": "u16", "char": "c_char", "mc_ctx": "McCtx", "mc_qweights": "McQweights",
          "mc_sampling": "McSampling"}


def c_to_rust(t: str) -> str:
    """A C type -> its Rust FFI spelling. Reading the declarator left to
    right: `const` before the first `*` qualifies the base type, `const`
    after a `*` qualifies that pointer; a Rust pointer is `*const` when what
    it points to is const (so `void* const*` is `*const *mut c_void`)."""
    toks = re.findall(r"\*|\bconst\b|[A-Za-z_]\w*(?: [A-Za-z_]\w*)*", " ".join(t.split()))
    base_const, base, ptr_const = False, [], []   # ptr_const[i]: pointer i is itself const
    for tok in toks:
        if tok == "*":
            ptr_const.append(False)
        elif tok == "const":
            if ptr_const:
                ptr_const[-1] = True
            else:
                base_const = True
        else:
            base += [w for w in tok.split() if w != "const"]
    r = C_BASE[" ".join(base)]
    pointee_const = base_const
    for pc in ptr_const:
        r = f"*{'const' if pointee_const else 'mut'} {r}"
        pointee_const = pc
    return r


def header_protos():
    src = (ROOT / "include" / "molten_cuda.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"^\s*([\w ][\w \*]*?)\b(mc_\w+)\s*\(([^;]*?)\);", src,
                                      flags=re.M | re.S):
        params = []
        args = " ".join(args.split())
        if args and args != "void":
            for a in args.split(","):
                m = re.match(r"(.*?)(\w+)$", a.strip())
                params.append((m.group(2), c_to_rust(m.group(1))))
        out[name] = (c_to_rust(ret.strip()), params)
    return out


def rust_decls():
    src = (ROOT / "include" / "cuda.rs").read_text()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    out = {}
    for name, args, ret in re.findall(r"pub fn (mc_\w+)\((.*?)\)\s*->\s*([^;]+);", block,
                                      flags=re.S):
        params = []
        for a in [x.strip() for x in args.split(",") if x.strip()]:
            n, t = a.split(":", 1)
            params.append((n.strip(), " ".join(t.split())))
        out[name] = (" ".join(ret.split()), params)
    return out


def test_every_entry_point_is_declared_with_matching_types():
    h, r = header_protos(), rust_decls()
    assert len(h) >= 60
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name, (ret, params) in h.items():
        rret, rparams = r[name]
        assert rret == ret, (name, rret, ret)
        assert [t for _, t in rparams] == [t for _, t in params], (name, rparams, params)
        assert [n for n, _ in rparams] == [n for n, _ in params], name


def test_structs_and_constants_agree():
    h = (ROOT / "include" / "molten_cuda.h").read_text()
    rs = (ROOT / "include" / "cuda.rs").read_text()
    for name, val in re.findall(r"#define (MC_[A-Z0-9_]+) \(?(-?\d+)\)?", h):
        m = re.search(rf"pub const {name}: c_int = (-?\d+);", rs)
        assert m and int(m.group(1)) == int(val), name
    for cname, rname in (("mc_qweights", "McQweights"), ("mc_sampling", "McSampling")):
        cbody = re.search(rf"typedef struct {cname} \{{(.*?)\}} {cname};", h, re.S).group(1)
        rbody = re.search(rf"pub struct {rname} \{{(.*?)\}}", rs, re.S).group(1)
        cf = re.findall(r"([\w ]+?\**)\s*(\w+);", cbody)
        rf = re.findall(r"pub (\w+): ([^,]+),", rbody)
        assert [n for _, n in cf] == [n for n, _ in rf], cname
        assert [c_to_rust(t) for t, _ in cf] == [" ".join(t.split()) for _, t in rf], cname
