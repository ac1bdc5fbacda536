"""adapters"""
