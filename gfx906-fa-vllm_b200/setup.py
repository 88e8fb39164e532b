"""Packaging for the sm_100a gfx906_fa plugin.

    python gfx906_fa_build.py          # build libgfx906fa_b200.so + gfx906_fa.so in place
    pip install -e .                   # register the vLLM plugin entry point

vLLM then loads `gfx906_fa_backend:register` in every process through the
`vllm.general_plugins` entry point, which registers the backend as
AttentionBackendEnum.CUSTOM (select it with --attention-backend CUSTOM).
"""
from setuptools import setup

setup(
    name="gfx906_fa",
    version="0.1.0",
    py_modules=["gfx906_fa_backend", "gfx906_fa_paged", "gfx906_fa_build"],
    package_data={"": ["gfx906_fa.so", "libgfx906fa_b200.so"]},
    entry_points={
        "vllm.general_plugins": [
            "gfx906_fa = gfx906_fa_backend:register",
        ],
    },
)
