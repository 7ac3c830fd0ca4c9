"""emmy.compiler.ir.kernel stand-in."""
