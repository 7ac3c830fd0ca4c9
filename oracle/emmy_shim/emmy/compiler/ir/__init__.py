"""emmy.compiler.ir stand-in."""
