"""daemon"""
