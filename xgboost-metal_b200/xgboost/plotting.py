"""Plotting (python-package/xgboost/plotting.py in the reference): feature
importance bars with matplotlib and trees through graphviz, both imported
only when called."""
import numpy as np

from .core import Booster

__all__ = ["plot_importance", "plot_tree", "to_graphviz"]


def _booster(model):
    if isinstance(model, Booster):
        return model
    if hasattr(model, "get_booster"):
        return model.get_booster()
    if isinstance(model, dict):
        return model
    raise ValueError("tree must be Booster, XGBModel or dict instance")


def plot_importance(booster, ax=None, height=0.2, xlim=None, ylim=None, title="Feature importance",
                    xlabel="Importance score", ylabel="Features", fmap="", importance_type="weight",
                    max_num_features=None, grid=True, show_values=True, values_format="{v}", **kwargs):
    """Horizontal bars of get_score(importance_type), largest at the top."""
    import matplotlib.pyplot as plt
    b = _booster(booster)
    importance = b if isinstance(b, dict) else b.get_score(fmap=fmap, importance_type=importance_type)
    if not importance:
        raise ValueError("Booster.get_score() results in empty.  This maybe caused by having all trees as "
                         "decision dumps.")
    items = sorted(importance.items(), key=lambda kv: kv[1])
    if max_num_features is not None:
        items = items[-max_num_features:]
    labels, values = zip(*items)
    if ax is None:
        _, ax = plt.subplots(1, 1)
    ylocs = np.arange(len(values))
    ax.barh(ylocs, values, align="center", height=height, **kwargs)
    if show_values:
        for x, y in zip(values, ylocs):
            ax.text(x + 1, y, values_format.format(v=x), va="center")
    ax.set_yticks(ylocs)
    ax.set_yticklabels(labels)
    ax.set_xlim(xlim if xlim is not None else (0, max(values) * 1.1))
    ax.set_ylim(ylim if ylim is not None else (-1, len(values)))
    if title is not None:
        ax.set_title(title)
    if xlabel is not None:
        ax.set_xlabel(xlabel)
    if ylabel is not None:
        ax.set_ylabel(ylabel)
    ax.grid(grid)
    return ax


def to_graphviz(booster, fmap="", num_trees=0, rankdir=None, yes_color=None, no_color=None,
                condition_node_params=None, leaf_node_params=None, with_stats=False, tree_idx=None,
                **kwargs):
    """One tree as a graphviz.Source of the library's dot dump."""
    from graphviz import Source
    b = _booster(booster)
    index = tree_idx if tree_idx is not None else num_trees
    dumps = b.get_dump(fmap=fmap, with_stats=with_stats, dump_format="dot")
    if not 0 <= index < len(dumps):
        raise IndexError("tree index %d out of range" % index)
    text = dumps[index]
    if rankdir is not None:
        text = text.replace("rankdir=TB", "rankdir=%s" % rankdir)
    return Source(text, **kwargs)


def plot_tree(booster, fmap="", num_trees=0, rankdir=None, ax=None, with_stats=False, tree_idx=0,
              **kwargs):
    """Draws one tree (rendered by graphviz as PNG) on matplotlib axes."""
    from io import BytesIO

    import matplotlib.image as image
    import matplotlib.pyplot as plt
    if ax is None:
        _, ax = plt.subplots(1, 1)
    g = to_graphviz(booster, fmap=fmap, rankdir=rankdir, with_stats=with_stats,
                    tree_idx=tree_idx or num_trees, **kwargs)
    img = image.imread(BytesIO(g.pipe(format="png")))
    ax.imshow(img)
    ax.axis("off")
    return ax

