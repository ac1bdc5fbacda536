"""scheduler"""
