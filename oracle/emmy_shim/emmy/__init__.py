"""Import shim: the ``emmy`` module surface the reference compiler imports.

The reference (``ptxc/``, ``compile.py``) depends on ``emmy-ml==0.3.11``,
which is not installed and not installable offline.  These modules expose this
repository's clean-room IR classes (``emmy_ir``) under the import paths the
reference uses, so the unmodified reference compiler can emit its PTX here --
as an oracle and a timing baseline only (test infrastructure).
"""
