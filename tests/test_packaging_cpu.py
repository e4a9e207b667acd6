"""Packaging metadata: the version comes from the package, both import names (the B200 package
and the ``flextensor`` facade) are packaged, and the CUDA sources ship with them."""

import os
import tomllib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pyproject_packages_and_version():
    with open(os.path.join(ROOT, "pyproject.toml"), "rb") as f:
        meta = tomllib.load(f)
    assert meta["project"]["dynamic"] == ["version"]
    assert meta["tool"]["setuptools"]["dynamic"]["version"]["attr"] == "flextensor_b200._version.__version__"
    inc = meta["tool"]["setuptools"]["packages"]["find"]["include"]
    assert "flextensor_b200*" in inc and "flextensor" in inc
    data = meta["tool"]["setuptools"]["package-data"]["flextensor_b200"]
    assert "ops/csrc/*.cu" in data and "ops/_build/*.so" in data
    import flextensor_b200

    assert flextensor_b200.__version__
    deps = " ".join(meta["project"]["dependencies"])
    for d in ("torch", "pydantic", "numpy", "scipy", "psutil"):
        assert d in deps
