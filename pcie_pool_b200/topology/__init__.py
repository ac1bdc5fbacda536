"""topology"""
