"""Import helper: the package directory name contains hyphens, so it is imported by name."""
import importlib

PKG_NAME = "flashattention-gpt-oss-finetuning_b200"


def pkg():
    return importlib.import_module(PKG_NAME)


def submodule(name):
    return importlib.import_module(f"{PKG_NAME}.{name}")
