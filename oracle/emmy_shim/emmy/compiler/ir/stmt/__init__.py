from emmy.compiler._model import Stmt  # noqa: F401
