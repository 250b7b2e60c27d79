"""Local repair, event-column selection and resynthesis branches."""
