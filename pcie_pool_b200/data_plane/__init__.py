"""data_plane"""
