"""worker"""
