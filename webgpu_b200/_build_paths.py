"""Where the in-tree native builds live (built by webgpu_b200.build, shipped with the tree)."""
import os

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PACKAGE_DIR)
BUILD_DIR = os.path.join(PACKAGE_DIR, "_build")


def wgd_lib_path() -> str:
    """The CUDA decoder library (C ABI declared in include/wgd.h)."""
    return os.environ.get("WGD_LIBRARY", os.path.join(BUILD_DIR, "libwgd.so"))


def synth_lib_path() -> str:
    """The seeded synthetic-weight generator (host code only)."""
    return os.path.join(BUILD_DIR, "libwgdsynth.so")


def oracle_lib_path() -> str:
    """The CPU oracle (test infrastructure; built from oracle/)."""
    return os.path.join(REPO_DIR, "oracle", "_build", "liboracle.so")
