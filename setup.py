"""`python setup.py build_ext --inplace`: builds this package's native parts in place, for sm_100a
-- lib/libdecode_rope.so (the C ABI library) and cuda/_ext*.so (the PyTorch binding) -- exactly
as `python -m decode_llm_kernel_b200._build` does. It is the build command the reference's
extension documents (its setup.py BUILD_COMMAND), so callers that print or check it keep
working when they load this package through the drop-in shim. It builds in place and does not
package the project.
"""
from setuptools import setup
from setuptools.command.build_ext import build_ext


class BuildInPlace(build_ext):
    def run(self):
        from decode_llm_kernel_b200 import _build
        _build.build()


if __name__ == "__main__":
    setup(name="decode_llm_kernel_b200", packages=[], py_modules=[],
          cmdclass={"build_ext": BuildInPlace})
