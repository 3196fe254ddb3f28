"""prism_cp_b200: Blackwell-native dynamic context-parallel training of hybrid GDN:GQA decoders."""

__version__ = "0.1.0"
