"""Packaging hook: `pip install .` first runs `make` so that libugdr.so, the daemon and the tools
exist in ugdr_b200/_lib/, then ships them as package data (metadata lives in pyproject.toml)."""
import os
import subprocess

from setuptools import setup
from setuptools.command.build_py import build_py


class BuildWithMake(build_py):
    def run(self):
        subprocess.check_call(["make", "-j"], cwd=os.path.dirname(os.path.abspath(__file__)))
        super().run()


# setuptools' own staging goes under build/py so it stays apart from the make objects (build/obj).
setup(cmdclass={"build_py": BuildWithMake},
      options={"build": {"build_base": "build/py"}, "egg_info": {"egg_base": "build/py"}})
