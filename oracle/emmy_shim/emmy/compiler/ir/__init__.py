"""``emmy.compiler.ir`` for the reference compiler."""
