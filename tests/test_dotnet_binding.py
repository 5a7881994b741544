"""The C# binding (project-ai_b200/dotnet/ProjectAI.Backends.Cuda) against the C ABI it binds, without a .NET SDK:

* every pai_* entry point that include/projectai_cuda.h declares has exactly one LibraryImport in Native.cs, with the
  same parameter count and the C#-side type each C parameter type maps to;
* CudaComputeBackend.cs implements every member of IComputeBackend (ProjectAI.Core/IComputeBackend.cs:9-96) and calls
  each import at least once;
* the registration patch adds the backend to the catalog and factory of ProjectAI/Backends.cs:13-31.
"""
import re

from conftest import ROOT

HEADER = ROOT / "include" / "projectai_cuda.h"
DOTNET = ROOT / "project-ai_b200" / "dotnet"
NATIVE = DOTNET / "ProjectAI.Backends.Cuda" / "Native.cs"
BACKEND = DOTNET / "ProjectAI.Backends.Cuda" / "CudaComputeBackend.cs"
PATCH = DOTNET / "Backends.cs.patch"

# C parameter type -> C# parameter type of the import
C_TO_CS = [
    (r"^(const )?pai_tensor\*$", "PaiTensor*"), (r"^pai_ctx\*$", "IntPtr"), (r"^pai_ctx\*\*$", "IntPtr*"),
    (r"^pai_graph\*$", "IntPtr"), (r"^pai_graph\*\*$", "IntPtr*"), (r"^(const )?float\*$", "float*"),
    (r"^(const )?int32_t\*$", "int*"), (r"^(const )?int64_t\*$", "long*"), (r"^double\*$", "double*"),
    (r"^(const )?uint8_t$", "byte*"), (r"^const void\*$", "IntPtr"), (r"^(const )?char\*$", "byte*"),
    (r"^(int32_t|int)$", "int"), (r"^int64_t$", "long"), (r"^float$", "float"),
]

# IComputeBackend members (IComputeBackend.cs:11-95)
CONTRACT = ["Name", "Device", "Allocate", "FromHost", "ToHost", "Copy", "Add", "Mul", "Sub", "Div", "AddScalar",
            "MulScalar", "Sqrt", "Sigmoid", "MatMul", "Sum", "Mean", "Max", "Softmax", "RmsNorm", "Silu",
            "RotaryEmbedding", "Gather", "ScatterAddRows", "CrossEntropy", "CrossEntropyGrad", "Cat", "BeginScope",
            "KeepAlive", "Release", "Dispose"]


def header_protos():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for name, args in re.findall(r"(?:const\s+)?\w+\*?\s+\*?(pai_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = [] if args.strip() == "void" else [" ".join(a.split()) for a in args.split(",")]
        out[name] = params
    return out


def imports():
    text = NATIVE.read_text()
    found = re.findall(r'\[LibraryImport\(Lib, EntryPoint = "(pai_[a-z0-9_]+)"\)\]\s*internal static partial (\w+) (\w+)\(([^)]*)\);',
                       text)
    return [(entry, ret, method, [p.strip() for p in params.split(",")] if params.strip() else [])
            for entry, ret, method, params in found]


def test_every_entry_point_has_exactly_one_import_with_matching_types():
    protos = header_protos()
    imps = imports()
    entries = [e for e, *_ in imps]
    assert sorted(entries) == sorted(protos), (set(protos) ^ set(entries))
    assert len(entries) == len(set(entries)), "an entry point is imported twice"
    for entry, ret, method, params in imps:
        cparams = protos[entry]
        assert len(params) == len(cparams), f"{entry}: {len(params)} C# parameters for {len(cparams)} C parameters"
        assert ret == ("IntPtr" if entry == "pai_last_error" else "int"), entry
        for c, cs in zip(cparams, params):
            ctype = re.sub(r"\s*\w+(\[128\])?$", "", c).strip()
            want = next((t for pat, t in C_TO_CS if re.match(pat, ctype)), None)
            assert want is not None, f"{entry}: unmapped C type {ctype!r}"
            assert cs.split()[0] == want, f"{entry}: C parameter {c!r} bound as {cs!r}, expected {want}"


def test_backend_implements_the_contract_and_uses_every_import():
    text = BACKEND.read_text()
    assert re.search(r"class CudaComputeBackend\s*:\s*IComputeBackend", text)
    for member in CONTRACT:
        assert re.search(rf"public [\w<>(),? .]+\b{member}\b", text), f"IComputeBackend.{member} is not implemented"
    for _, _, method, _ in imports():
        if method == "LastError":
            continue
        assert f"Native.{method}(" in text, f"Native.{method} is never called"


def test_registration_patch_adds_catalog_entry_and_factory_branch():
    patch = PATCH.read_text()
    added = "\n".join(line[1:] for line in patch.splitlines() if line.startswith("+") and not line.startswith("+++"))
    assert "using ProjectAI.Backends.Cuda;" in added
    assert 'new("cuda",' in added
    assert "new CudaComputeBackend(" in added
    assert "CudaComputeBackend.IsAvailable(" in added
