"""include/nmg.hpp compiles as C++20 against libnmg.so and maps statuses onto the reference's exceptions."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_header_builds_and_maps_errors(tmp_path):
    exe = tmp_path / "nmg_hpp_check"
    src = os.path.join(ROOT, "tests", "cpp", "nmg_hpp_check.cpp")
    lib = os.path.join(ROOT, "hero_b200")
    subprocess.run(["g++", "-std=c++20", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), src,
                    "-L", lib, "-lnmg", f"-Wl,-rpath,{lib}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("PASS") == 5 and "FAIL" not in r.stdout
