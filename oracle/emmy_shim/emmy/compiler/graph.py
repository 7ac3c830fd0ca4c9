from emmy.compiler._model import Graph, Node  # noqa: F401
