"""``emmy.compiler`` for the reference compiler (see ``emmy/__init__.py``)."""
