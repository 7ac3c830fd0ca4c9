from emmy.compiler._model import Accum, Assign, Init, Let, Load, Write  # noqa: F401
