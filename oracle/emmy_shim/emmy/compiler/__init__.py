"""emmy.compiler stand-in."""
