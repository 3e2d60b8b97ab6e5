"""The Java (FFM) binding under integration/java against the C ABI it binds
(no JDK needed): every prototype of include/jax4j_cuda.h has exactly one
downcall handle in J4C.java whose FunctionDescriptor matches it (C int /
int32_t / uint32_t -> JAVA_INT, int64_t / uint64_t / size_t -> JAVA_LONG,
double -> JAVA_DOUBLE, float -> JAVA_FLOAT, pointers, streams and
communicators -> ADDRESS), every invokeExact call site passes as many
arguments as its prototype takes, and CudaBackend implements every method of
the reference's ExecutionBackend (backend/ExecutionBackend.java:11-56)."""
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]
JAVA = ROOT / "integration" / "java" / "com" / "marmanis" / "jax4j" / "backend" / "cuda"
HEADER = ROOT / "include" / "jax4j_cuda.h"

SCALARS = {"int": "JAVA_INT", "int32_t": "JAVA_INT", "uint32_t": "JAVA_INT", "int64_t": "JAVA_LONG",
           "uint64_t": "JAVA_LONG", "size_t": "JAVA_LONG", "double": "JAVA_DOUBLE", "float": "JAVA_FLOAT"}


def _layout(ctype: str) -> str:
    t = " ".join(ctype.split())
    if "*" in t or t.split()[-1] in ("j4c_stream", "j4c_comm"):
        return "ADDRESS"
    return SCALARS[t.replace("const ", "").strip()]


def header_prototypes():
    src = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"J4C_API\s+([^;]+?)\s*\(([^;]*?)\)\s*;", src, flags=re.S):
        head, args = " ".join(m.group(1).split()), " ".join(m.group(2).split())
        name = re.findall(r"(\w+)$", head)[0]
        ret = head[: -len(name)].strip()
        params = [] if args == "void" else [_layout(re.sub(r"\s*\b\w+$", "", a.strip())) for a in args.split(",")]
        out[name] = (None if ret == "void" else _layout(ret), params)
    return out


def java_handles():
    src = (JAVA / "J4C.java").read_text()
    out = {}
    pat = r"MethodHandle\s+(\w+)\s*=\s*h\(\s*\"(\w+)\"\s*,\s*FunctionDescriptor\.(of|ofVoid)\(([^;]*?)\)\s*\)\s*;"
    for m in re.finditer(pat, src, flags=re.S):
        const, name, kind, args = m.groups()
        layouts = [a.strip() for a in args.split(",") if a.strip()]
        assert name not in out, f"{name} bound twice"
        out[name] = (const, (layouts[0] if kind == "of" else None), layouts[1:] if kind == "of" else layouts)
    return out


def test_header_parses():
    protos = header_prototypes()
    assert len(protos) >= 70 and "j4c_dot_split_ep_bits" in protos and "j4c_psum" in protos


def test_every_entry_point_is_bound_with_a_matching_descriptor():
    protos, handles = header_prototypes(), java_handles()
    assert set(protos) == set(handles), (sorted(set(protos) - set(handles)), sorted(set(handles) - set(protos)))
    for name, (ret, params) in protos.items():
        _, jret, jparams = handles[name]
        assert jret == ret, f"{name}: returns {ret}, Java binds {jret}"
        assert jparams == params, f"{name}: C ({', '.join(params)}) vs Java ({', '.join(jparams)})"


def _top_level_args(s: str) -> int:
    depth, n = 0, 1
    if not s.strip():
        return 0
    for ch in s:
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        elif ch == "," and depth == 0:
            n += 1
    return n


def test_call_sites_pass_every_argument():
    protos, handles = header_prototypes(), java_handles()
    by_const = {c: name for name, (c, _, _) in handles.items()}
    calls = 0
    for f in JAVA.glob("*.java"):
        src = f.read_text()
        for m in re.finditer(r"J4C\.(\w+)\.invokeExact\(", src):
            const = m.group(1)
            assert const in by_const, f"{f.name}: J4C.{const} is not a bound handle"
            i, depth = m.end(), 1
            while depth:
                depth += {"(": 1, ")": -1}.get(src[i], 0)
                i += 1
            n = _top_level_args(src[m.end():i - 1])
            want = len(protos[by_const[const]][1])
            assert n == want, f"{f.name}: J4C.{const}.invokeExact passes {n} arguments, the C function takes {want}"
            calls += 1
    assert calls >= 20


def test_cuda_backend_implements_execution_backend():
    src = (JAVA / "CudaBackend.java").read_text()
    assert "implements ExecutionBackend" in src
    # backend/ExecutionBackend.java:11-56: four float[] methods, four double[] defaults
    wanted = [r"float\[\]\s+binary\(Primitive \w+, float\[\] \w+, float\[\] \w+, Device \w+\)",
              r"float\[\]\s+unary\(Primitive \w+, float\[\] \w+, Device \w+\)",
              r"float\[\]\s+matmul\(float\[\] \w+, float\[\] \w+, int \w+, int \w+, int \w+, Device \w+\)",
              r"float\[\]\s+reduce\(Primitive \w+, float\[\] \w+, Device \w+\)",
              r"double\[\]\s+reduce\(Primitive \w+, double\[\] \w+, Device \w+\)",
              r"double\[\]\s+binary\(Primitive \w+, double\[\] \w+, double\[\] \w+, Device \w+\)",
              r"double\[\]\s+unary\(Primitive \w+, double\[\] \w+, Device \w+\)",
              r"double\[\]\s+matmul\(double\[\] \w+, double\[\] \w+, int \w+, int \w+, int \w+, Device \w+\)"]
    for w in wanted:
        assert re.search(r"@Override\s+public\s+" + w, src), f"CudaBackend lacks {w}"


def test_collective_replacement_mirrors_shared_collective():
    src = (JAVA / "CudaCollective.java").read_text()
    # api/SharedCollective.java:44 and :60 -- the two operations PmapContext's users call
    assert re.search(r"public float\[\] psum\(int deviceIndex, float\[\] data\)", src)
    assert re.search(r"public DeviceStorage allGather\(int deviceIndex, DeviceStorage shard\)", src)
    assert "barrier.await(timeoutMs" in src  # bounded, unlike CyclicBarrier.await()


def test_fused_program_struct_offsets_match_the_c_layout():
    """CudaFusedProgram writes j4c_insn / j4c_program at the offsets the C
    struct has (natural alignment: the ctypes mirror in fusion.py, which
    fused.cu's static_asserts pin to the header)."""
    import ctypes
    from jax4j_b200 import fusion
    src = (JAVA / "CudaFusedProgram.java").read_text()
    prog_sets = re.findall(r"prog\.set\((JAVA_INT|ADDRESS), (\d+),", src)
    fields = [f for f, _ in fusion._Program._fields_]
    want = [getattr(fusion._Program, f).offset for f in fields]
    assert [int(o) for _, o in prog_sets] == want, (prog_sets, list(zip(fields, want)))
    kinds = ["JAVA_INT" if t is ctypes.c_int32 else "ADDRESS" for _, t in fusion._Program._fields_]
    assert [k for k, _ in prog_sets] == kinds
    assert ctypes.sizeof(fusion._Program) == 80
    insn_sets = re.findall(r"e\.set\((JAVA_INT|JAVA_DOUBLE), (\d+),", src)
    assert [int(o) for _, o in insn_sets] == [getattr(fusion._Insn, f).offset for f, _ in fusion._Insn._fields_]
    assert ctypes.sizeof(fusion._Insn) == 24
