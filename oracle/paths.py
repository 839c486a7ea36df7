"""TEST INFRASTRUCTURE ONLY -- where the reference source tree is.

The reference tree exists only in the build container.  Its location comes
from the REF_ROOT environment variable (the same variable oracle/Makefile
reads), with the build container's path as the default.  Only the fixture
generators under tests/golden/ and the build step of the oracle read it;
nothing that runs on a GPU box does.
"""
import os

REF_ROOT = os.environ.get("REF_ROOT", "/root/reference")
