"""Dataset registry (reference: t10n/dataset/meta.py:1-174).

Same names and shapes as the reference.  ``name_to_meta`` also accepts
``rmat_<scale>`` names (the reference checks a list without them first,
t10n/dataset/meta.py:152-153, so its rmat branch is unreachable) and the seeded
synthetic specs of grappa_b200.dataset.synthetic.
"""


class _Meta:
    def __init__(self, name, origin_name, n_n, n_e, origin_n_e, n_dim, n_label, origin_path):
        self.name, self.origin_name = name, origin_name
        self.n_n, self.n_e, self.origin_n_e = n_n, n_e, origin_n_e
        self.n_dim, self.n_label = n_dim, n_label
        self.origin_path = origin_path

    def __repr__(self):
        return f"meta({self.name}: {self.n_n} nodes, {self.n_e} edges, dim {self.n_dim}, {self.n_label} classes)"


def reddit_meta():
    return _Meta("reddit", "reddit", 232965, 114848857, 114615892, 602, 41, "reddit")


def ogbpr_meta():
    return _Meta("ogbpr", "ogbn-products", 2449029, 126167053, 61859140, 100, 47, "ogbn_products/raw")


def ogbar_meta():
    return _Meta("ogbar", "ogbn-arxiv", 169343, 1335586, 1166243, 128, 40, "ogbn_arxiv/raw")


def ogbpa_meta():
    return _Meta("ogbpa", "ogbn-papers100M", 111059956, 1726745828, 1615685872, 128, 172, "ogbn_papers100M/raw")


def cora_meta():
    return _Meta("cora", "cora", 2708, 13264, 10556, 1433, 7, "cora_v2")


def igb_meta():
    return _Meta("igb260m", "igb260m", 269346174, 3727095830, 3727095830, 1024, 19,
                 "igb/IGB-Datasets/igb/igb-public.s3.us-east-2.amazonaws.com/IGBH/processed/")


def mag_meta():
    return _Meta("mag", "mag240m", 244160499, 1728364232, 1728364232, 768, 349, "mag240m")


def rmat_meta(scale=26):
    n = 2 ** scale
    return _Meta(f"rmat_{scale}", f"rmat_{scale}", n, 2 ** (scale + 4), 2 ** (scale + 4), 128, 19, "rmat")


_TABLE = {"reddit": reddit_meta, "ogbpr": ogbpr_meta, "ogbar": ogbar_meta, "ogbpa": ogbpa_meta,
          "cora": cora_meta, "igb260m": igb_meta, "mag": mag_meta}


def name_to_meta(name: str):
    if name in _TABLE:
        return _TABLE[name]()
    if name.startswith("rmat_"):
        return rmat_meta(int(name.split("_")[1]))
    from grappa_b200.dataset.synthetic import SPECS

    if name in SPECS:
        s = SPECS[name]
        return _Meta(name, name, s.n_nodes, 2 * s.n_edges + s.n_nodes, 2 * s.n_edges, s.feat_dim, s.n_classes,
                     "synthetic")
    raise AssertionError(f"dataset {name} in not supported")


def t10n_chunk_path(dataset_name, part_method, n_part):
    return f"chunking_{dataset_name}_{part_method}_{n_part:03}"
