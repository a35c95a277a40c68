"""CPU checks of the Rust binding (vestra-kernels_b200/bindings/rust): the
record layouts it mirrors, asserted by a C program compiled against the
header, and its extern block declaring exactly the header's entry points.
There is no Rust toolchain here, so the binding itself is not compiled."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vestra_b200.h")
FFI = os.path.join(ROOT, "vestra-kernels_b200", "bindings", "rust", "src", "b200", "ffi.rs")


def test_c_record_layouts(tmp_path):
    exe = tmp_path / "abi_layout"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "abi_layout.c"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def _header_functions():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return re.findall(r"\n(?:int|const char\*)\s+(vk_\w+)\s*\(", src)


def test_rust_ffi_declares_every_entry_point():
    src = open(FFI).read()
    rust = re.findall(r"pub fn (vk_\w+)\(", src)
    assert rust == _header_functions()


def test_rust_ffi_argument_counts():
    hdr = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    protos = dict(re.findall(r"\n(?:int|const char\*)\s+(vk_\w+)\s*\(([^;]*)\);", hdr))
    for name, args in re.findall(r"pub fn (vk_\w+)\(([^)]*)\)", open(FFI).read()):
        c_args = protos[name].strip()
        n_c = 0 if c_args in ("", "void") else c_args.count(",") + 1
        n_rs = 0 if not args.strip() else args.count(",") + 1
        assert n_c == n_rs, name
