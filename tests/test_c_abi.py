"""libtrmoe.so from C: tests/c/abi_test.c, compiled as strict C11 against include/trmoe.h together with a table of
every declared function's address (so a declaration the library does not export fails to link), run without a GPU
(the conventions: NULL contexts with messages, host-only answers). tests/test_gpu_c_abi.py runs the
same program's GPU part."""
import os
import subprocess

from tests.test_capi import declared_functions

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_abi_test(out_dir) -> str:
    from trochilus_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()
    refs = os.path.join(str(out_dir), "refs.c")
    with open(refs, "w") as f:
        f.write('#include "trmoe.h"\ntypedef void (*trmoe_fn)(void);\nconst trmoe_fn trmoe_abi_refs[] = {\n')
        f.write("".join(f"    (trmoe_fn){n},\n" for n in declared_functions()))
        f.write("};\n")
    exe = os.path.join(str(out_dir), "abi_test")
    lib_dir, orc_dir = os.path.join(ROOT, "trochilus_b200"), os.path.join(ROOT, "oracle")
    subprocess.check_call(["gcc", "-std=c11", "-O1", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I",
                           os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "c", "abi_test.c"), refs,
                           f"-L{lib_dir}", "-ltrmoe", f"-L{orc_dir}", "-loracle", f"-Wl,-rpath,{lib_dir}",
                           f"-Wl,-rpath,{orc_dir}", "-lm", "-o", exe])
    return exe


def test_c_abi_without_gpu(tmp_path):
    exe = build_abi_test(tmp_path)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "cpu ok", (out.returncode, out.stdout, out.stderr)
